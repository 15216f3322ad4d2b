"""Pre-norm hybrid MoE transformer (model/transformer.py:27-417).

Block: ``x += rs * attn(norm1(x)); x += rs * ffn(norm2(x))`` with ONE
learnable residual scale per block shared by both adds (transformer.py:80-99),
fp32 residual stream, per-layer attention type (full / swa / kda), dense FFN
for the first ``dense_layers`` layers and MoE after, tied fp32-master
embedding used as the output head.
"""
from __future__ import annotations

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint

from .. import ops
from ..config import Config
from ..ops import reference as ref
from ..utils.nvtx import rng
from .layers import KDA, Attention, DenseFFN, MoE, RMSNorm


class _UnitBoundary(torch.autograd.Function):
    """Identity on the tensors that cross a unit (block) boundary.  Its
    backward runs ``cb``: placed at a block's input it fires once every
    gradient of that block is final; at a block's output, just before the
    block's backward starts.  The engine uses the first to launch the block's
    gradient reduce-scatter while the backward of earlier blocks continues."""

    @staticmethod
    def forward(ctx, cb, *xs):
        ctx.cb = cb
        return xs

    @staticmethod
    def backward(ctx, *gs):
        ctx.cb()
        return (None,) + gs


def unit_boundary(hooks, event: str, unit: int, *xs):
    """Route ``xs`` through a boundary whose backward calls
    ``hooks.<event>(unit)``; a no-op without hooks or outside autograd."""
    if hooks is None or not torch.is_grad_enabled() or not any(x.requires_grad for x in xs):
        return xs
    return _UnitBoundary.apply(lambda: getattr(hooks, event)(unit), *xs)


class Block(nn.Module):
    def __init__(self, cfg: Config, layer: int, gen: torch.Generator, ep=None):
        super().__init__()
        self.layer = layer
        self.attention_type = cfg.layer_types()[layer]
        self.use_moe = layer >= cfg.dense_layers
        self.norm1 = RMSNorm(cfg.d_model, cfg.norm_eps)
        if self.attention_type == "kda":
            self.attn = KDA(cfg.d_model, cfg.kda_heads, cfg.kda_head_dim, gen,
                            chunk=cfg.kda_chunk_size, gate=cfg.kda_gate)
        else:
            self.attn = Attention(cfg.d_model, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, gen,
                                  window=cfg.layer_window(layer))
        self.norm2 = RMSNorm(cfg.d_model, cfg.norm_eps)
        if self.use_moe:
            self.ffn = MoE(cfg.d_model, cfg.d_ff, cfg.n_experts, cfg.n_active,
                           cfg.n_shared_experts, cfg.router_init_std, cfg.routed_scaling_factor,
                           gen, d_ff_shared=cfg.d_ff_shared, router_type=cfg.router_type, ep=ep)
        else:
            self.ffn = DenseFFN(cfg.d_model, cfg.d_ff_shared, gen)
        self.residual_scale = nn.Parameter(torch.tensor(float(cfg.residual_scale_init)))

    def mix(self, h, cos, sin, dtype, positions=None, cache=None):
        """Token mixer (attention or KDA) on the normed input."""
        if self.attention_type == "kda":
            return self.attn(h, dtype, state=None if cache is None else cache.kda_state(self.layer))
        return self.attn(h, cos, sin, dtype, positions=positions,
                         cache=None if cache is None else cache.kv(self.layer))

    def feed_forward(self, h, dtype):
        if self.use_moe:
            return self.ffn(h, dtype)
        return self.ffn(h, dtype), {}

    def _mixer_half(self, x, cos, sin, dtype, positions=None, cache=None):
        h = self.norm1(x, dtype)
        a = self.mix(h, cos, sin, dtype, positions, cache)
        return x + self.residual_scale.float() * a

    def _ffn_half(self, x, dtype):
        h = self.norm2(x, dtype)
        f, aux = self.feed_forward(h, dtype)
        return x + self.residual_scale.float() * f, aux

    def _whole(self, x, cos, sin, dtype, positions=None):
        return self._ffn_half(self._mixer_half(x, cos, sin, dtype, positions), dtype)

    def forward(self, x, cos, sin, dtype, positions=None, cache=None, remat="none"):
        if remat == "full" and cache is None and torch.is_grad_enabled():
            return checkpoint(self._whole, x, cos, sin, dtype, positions, use_reentrant=False)
        if remat == "experts" and cache is None and torch.is_grad_enabled():
            x = checkpoint(self._mixer_half, x, cos, sin, dtype, positions, use_reentrant=False)
        else:
            x = self._mixer_half(x, cos, sin, dtype, positions, cache)
        return self._ffn_half(x, dtype)


class Transformer(nn.Module):
    """Full model.  ``forward(tokens)`` returns the final normed hidden state
    (compute dtype) and the merged aux dict; :meth:`logits` applies the tied
    head.  Training uses :meth:`loss`, which fuses the head with the CE."""

    def __init__(self, cfg: Config, seed: int = 0, ep=None):
        """``ep = (rank, world)``: expert parallelism; each MoE layer keeps only
        this rank's experts as it is built (host memory stays at one layer's
        experts instead of the whole model's)."""
        super().__init__()
        self.cfg = cfg
        gen = torch.Generator().manual_seed(seed)
        std = cfg.d_model ** -0.5
        self.wte = nn.Parameter(torch.randn(cfg.vocab_size, cfg.d_model, generator=gen) * std)
        self.blocks = nn.ModuleList([Block(cfg, i, gen, ep=ep) for i in range(cfg.layers)])
        self.norm_f = RMSNorm(cfg.d_model, cfg.norm_eps)
        max_len = max(cfg.seq_len, cfg.infer_seq_len)
        cos, sin = ref.precompute_rope(cfg.head_dim, max_len, cfg.rope_base, cfg.yarn_factor,
                                       cfg.yarn_beta_fast, cfg.yarn_beta_slow)
        # RoPE tables are constants stored in the compute dtype (model/rope.py,
        # model/transformer.py:197-206), not parameters.
        dt = cfg.compute_dtype()
        self.register_buffer("rope_cos", cos.to(dt), persistent=False)
        self.register_buffer("rope_sin", sin.to(dt), persistent=False)
        self.n_moe = sum(1 for b in self.blocks if b.use_moe)
        # set by a data-parallel engine: post_backward(unit) / pre_backward(unit)
        # callbacks; unit i + 1 is block i (unit 0 is the embedding)
        self.unit_hooks = None

    @property
    def dtype(self):
        return self.cfg.compute_dtype()

    def embed(self, tokens):
        if tokens.is_cuda:
            from ..ops.norm import embedding_cuda
            return embedding_cuda(tokens, self.wte)
        return self.wte[tokens].float()

    def remat_policy(self) -> str:
        """Activation recompute of the training forward (model/transformer.py:100-181):
        ``full`` recomputes each block in its backward (only the block input is
        kept); ``experts`` recomputes the token mixer and keeps the MoE / FFN
        activations (the reference keeps the expert matmul outputs);
        ``dots`` / ``dots_no_batch`` keep every projection output and recompute
        the KDA chunk intermediates, the model's largest activations; ``none``
        keeps everything.  ``remat=False`` is ``none``."""
        c = self.cfg
        return c.remat_policy if c.remat else "none"

    def _apply_core_recompute(self):
        core = self.remat_policy() in ("dots", "dots_no_batch")
        for b in self.blocks:
            if b.attention_type == "kda":
                b.attn.recompute_core = core

    def _fused_residual_ok(self, x, cache) -> bool:
        D = self.cfg.d_model
        return (x.is_cuda and cache is None and self.dtype == torch.bfloat16 and D % 4 == 0
                and D <= 2048)

    def _forward_fused(self, x, positions):
        """CUDA path: every residual add is fused with the RMSNorm that follows
        it (norm2 of the same block, norm1 of the next block, or norm_f)."""
        dtype = self.dtype
        aux_list = []
        h = self.blocks[0].norm1(x, dtype)
        remat = self.remat_policy() if torch.is_grad_enabled() else "none"
        hooks = self.unit_hooks
        for i, blk in enumerate(self.blocks):
            if hooks is not None:
                hooks.pre_forward(i + 1)
            x, h = unit_boundary(hooks, "post_backward", i + 1, x, h)
            if remat == "full":
                x, h, aux = checkpoint(self._fused_block, i, x, h, positions, use_reentrant=False)
            else:
                if remat == "experts":
                    x, h = checkpoint(self._fused_mixer, i, x, h, positions, use_reentrant=False)
                else:
                    x, h = self._fused_mixer(i, x, h, positions)
                x, h, aux = self._fused_ffn(i, x, h)
            x, h = unit_boundary(hooks, "pre_backward", i + 1, x, h)
            if hooks is not None:
                hooks.post_forward(i + 1)
            if aux:
                aux_list.append(aux)
        return h, merge_aux(aux_list, self.cfg.n_experts, self.n_moe, x.device)

    def _fused_mixer(self, i, x, h, positions):
        from ..ops.norm import add_rms_norm_cuda
        blk = self.blocks[i]
        with rng(f"layer{i}/{blk.attention_type}"):
            a = blk.mix(h, self.rope_cos, self.rope_sin, self.dtype, positions)
            return add_rms_norm_cuda(x, a, blk.residual_scale, blk.norm2.weight, blk.norm2.eps)

    def _fused_ffn(self, i, x, h):
        from ..ops.norm import add_rms_norm_cuda
        blk = self.blocks[i]
        with rng(f"layer{i}/{'moe' if blk.use_moe else 'ffn'}"):
            f, aux = blk.feed_forward(h, self.dtype)
            nxt = self.blocks[i + 1].norm1 if i + 1 < len(self.blocks) else self.norm_f
            x, h = add_rms_norm_cuda(x, f, blk.residual_scale, nxt.weight, nxt.eps)
        return x, h, aux

    def _fused_block(self, i, x, h, positions):
        x, h = self._fused_mixer(i, x, h, positions)
        return self._fused_ffn(i, x, h)

    def forward(self, tokens, positions=None, cache=None):
        dtype = self.dtype
        self._apply_core_recompute()
        if self.unit_hooks is not None:
            self.unit_hooks.pre_forward(0)   # the embedding (also the tied head)
        x = self.embed(tokens)
        if self._fused_residual_ok(x, cache):
            return self._forward_fused(x, positions)
        aux_list = []
        remat = self.remat_policy() if torch.is_grad_enabled() else "none"
        hooks = self.unit_hooks if cache is None else None
        for i, blk in enumerate(self.blocks):
            if self.unit_hooks is not None:
                self.unit_hooks.pre_forward(i + 1)
            (x,) = unit_boundary(hooks, "post_backward", i + 1, x)
            x, aux = blk(x, self.rope_cos, self.rope_sin, dtype, positions, cache, remat=remat)
            (x,) = unit_boundary(hooks, "pre_backward", i + 1, x)
            if self.unit_hooks is not None:
                self.unit_hooks.post_forward(i + 1)
            if aux:
                aux_list.append(aux)
        h = self.norm_f(x, dtype)
        return h, merge_aux(aux_list, self.cfg.n_experts, self.n_moe, x.device)

    def logits(self, h):
        """Tied fp32-accumulated head ``h @ wte^T`` (model/transformer.py:408-410)."""
        return ops.linear_t(h.reshape(-1, h.shape[-1]), self.wte).view(*h.shape[:-1], -1)

    def loss(self, tokens):
        """Total loss and metrics (train.py:180-217): CE over the full-length
        forward shifted by one, + z-loss + balance loss."""
        cfg = self.cfg
        h, aux = self(tokens)
        B, S, D = h.shape
        hs = h[:, :-1].reshape(B * (S - 1), D)
        tgt = tokens[:, 1:].reshape(-1)
        with rng("head_ce"):
            ce = ops.head_cross_entropy(hs, self.wte, tgt, compute_dtype=self.dtype)
        z = cfg.z_loss_weight * aux["router_z_loss"]
        bal = cfg.balance_loss_weight * aux["balance_loss"]
        total = ce + z + bal
        counts = aux["expert_counts"]
        share = counts / (counts.sum(-1, keepdim=True) + 1e-9)
        load_entropy = -(share * torch.log(share + 1e-9)).sum(-1)
        eff = torch.exp(load_entropy).mean()
        metrics = {"ce": ce.detach(), "z_loss": z.detach(), "bal_loss": bal.detach(),
                   "mean_entropy": aux["mean_entropy"].detach(), "eff_experts": eff.detach(),
                   "expert_counts": counts.detach()}
        return total, metrics

    def moe_layers(self):
        return [b.ffn for b in self.blocks if b.use_moe]


def merge_aux(aux_list, n_experts, n_moe, device):
    """Average scalar aux over MoE layers, stack expert counts [n_moe, N]
    (model/transformer.py:411-416)."""
    if not aux_list:
        z = torch.zeros((), device=device)
        return {"router_z_loss": z, "balance_loss": z, "mean_entropy": z,
                "expert_counts": torch.zeros(max(1, n_moe), n_experts, device=device)}
    n = max(1, n_moe)
    out = {}
    for k in ("router_z_loss", "balance_loss", "mean_entropy"):
        out[k] = torch.stack([a[k] for a in aux_list]).sum(0) / n
    out["expert_counts"] = torch.stack([a["expert_counts"] for a in aux_list])
    return out
