"""Configuration dataclass and presets.

Field names, defaults and the five reference presets (``smoke``, ``smoke_kda``,
``full``, ``full_g4``, ``custom``) follow the reference's ``config.py:13-323`` so
that a user of the reference finds the same knobs under the same names.  B200
additions (optimizer choice, router type, expert-parallel capacity, the KDA gate
parameterisation, micro-batching, fused-path toggles) are grouped at the end of
the dataclass, and the BASELINE benchmark configurations are added as presets
``tiny_hybrid``, ``hybrid_1p3b``, ``ep_moe``, ``long_kda``.
"""
from __future__ import annotations

import copy
from dataclasses import asdict, dataclass, fields
from typing import Optional


@dataclass
class Config:
    # ---- Model architecture (reference config.py:15-31) ----
    name: str = "smoke"
    vocab_size: int = 256
    layers: int = 2
    d_model: int = 64
    n_q_heads: int = 2
    n_kv_heads: int = 1
    head_dim: int = 32
    n_experts: int = 4
    n_active: int = 2
    n_shared_experts: int = 1
    d_ff: int = 128
    d_ff_dense: Optional[int] = None
    dense_layers: int = 1

    # ---- Norm ----
    norm_eps: float = 1e-6
    residual_scale_init: float = 1.0

    # ---- RoPE / YaRN ----
    rope_base: float = 10000.0
    yarn_factor: float = 1.0
    yarn_attn_factor: float = 1.0
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0

    # ---- MoE routing ----
    router_init_std: float = 0.01
    routed_scaling_factor: float = 2.5
    bias_update_rate: float = 0.001
    z_loss_weight: float = 1e-3
    balance_loss_weight: float = 1e-4
    n_group: int = 1

    # ---- Training ----
    batch_size: int = 2
    seq_len: int = 128
    train_steps: int = 10
    learning_rate: float = 1e-4
    min_lr: float = 1e-5
    warmup_steps: int = 2000
    decay_fraction: float = 0.2
    weight_decay: float = 1.0
    grad_clip: float = 1.0
    dtype: str = "bf16"
    master_dtype: str = "fp32"
    remat: bool = True
    remat_policy: str = "dots_no_batch"
    fused_step: bool = True
    opt_state_dtype: str = "bf16"

    # ---- Data ----
    dataset: str = "openbmb/Ultra-FineWeb-L3"
    dataset_config: Optional[str] = "Ultra-FineWeb-L3-en-Multi-Style-Synthetic"
    dataset_files: Optional[str] = (
        "hf://datasets/openbmb/Ultra-FineWeb-L3/"
        "data/ultrafineweb_en_l3/multi_style/*.parquet")
    tokenizer: str = "byte"
    pack_eos_id: Optional[int] = None

    # ---- Loader (the reference's Grain knobs; here a seeded synthetic /
    # parquet loader with the same buffering semantics) ----
    use_grain: bool = False
    grain_interleave: int = 4
    grain_cpu_buffer: int = 8
    grain_device_buffer: int = 2
    grain_shuffle_files: bool = True
    grain_seed: int = 0

    # ---- Hardware / sharding ----
    mesh_data_axis: int = 1
    mesh_expert_axis: int = 1
    checkpoint_every: int = 0
    checkpoint_dir: str = "checkpoints"

    # ---- Sliding-window hybrid ----
    use_swa: bool = False
    swa_window: int = 4096
    swa_period: int = 2

    # ---- KDA hybrid ----
    use_kda: bool = False
    kda_period: int = 4
    kda_heads: int = 64
    kda_head_dim: int = 128
    kda_chunk_size: int = 64
    use_scan: bool = True

    # ---- Inference ----
    infer_seq_len: int = 32768

    # ---- In-training sampling ----
    gen_every: int = 0
    gen_prompt: str = "The meaning of life is"
    gen_max_tokens: int = 40
    gen_temperature: float = 0.8
    gen_top_k: int = 40

    # ---- Logging ----
    log_every: int = 1
    # path of a JSON-lines metrics sink (one record per logged step; "" = off)
    metrics_jsonl: str = ""

    # ================= B200 additions =================
    # Optimizer: "lion" (reference parity, optimizer.py:126-155) or "adamw".
    optimizer: str = "lion"
    adam_b1: float = 0.9
    adam_b2: float = 0.95
    adam_eps: float = 1e-8
    lion_b1: float = 0.9
    lion_b2: float = 0.99
    # Router: "sigmoid_bias" (reference, moe.py:177-192) or "softmax"
    # (plain top-k softmax router, renormalised over the selected experts).
    router_type: str = "sigmoid_bias"
    # Switch-style load-balancing loss weight used by the softmax router.
    aux_loss_weight: float = 0.0
    # Expert-parallel token dispatch capacity (0 = dropless).
    capacity_factor: float = 0.0
    # KDA decay parameterisation: "kimi" is g = -exp(A_log)*softplus(f+dt_bias)
    # (reference kda.py:272-281); "sigmoid" is g = logsigmoid(f + dt_bias).
    kda_gate: str = "kimi"
    # Sequences per micro-batch inside one optimizer step (0 = whole batch).
    micro_batch: int = 0
    # Use the hand-written fused compute+collective paths when world > 1.
    fused_comm: bool = True
    # data parallelism: reduce-scatter each block's gradients during the last
    # micro-batch's backward, as soon as they are final (False: after the backward)
    overlap_reduce: bool = True
    # FSDP (ZeRO-3): with data parallelism the compute-dtype working copy of every
    # block's and the embedding's matrices is sharded over the ranks and gathered
    # for each use (forward, then again for the backward) into a buffer that is
    # freed afterwards (model/sharding.py:67-113); False keeps it replicated
    shard_params: bool = True
    # MoE expert weights under data parallelism (no expert axis): "replicated"
    # keeps the full bf16 working copy on every rank (the optimizer stores each
    # updated shard into every peer); "fused_gather" keeps only the rank's own
    # experts current and pulls the others inside the first grouped GEMM that
    # consumes them (all-gather fused with the GEMM, over peer memory).
    expert_weights: str = "replicated"
    seed: int = 0

    # ------------------------------------------------------------------
    def compute_dtype(self):
        import torch
        return {"bf16": torch.bfloat16, "fp32": torch.float32,
                "fp16": torch.float16}[self.dtype]

    def master_dtype_torch(self):
        import torch
        return {"fp32": torch.float32, "bf16": torch.bfloat16,
                "fp16": torch.float16}[self.master_dtype]

    @property
    def d_ff_shared(self) -> int:
        return self.d_ff if self.d_ff_dense is None else self.d_ff_dense

    def layer_types(self) -> list[str]:
        """Per-layer attention type, same priority rule as the reference
        (``model/transformer.py:238-250``): KDA outranks SWA."""
        out = []
        for i in range(self.layers):
            if self.use_kda:
                out.append("full" if i % self.kda_period == self.kda_period - 1 else "kda")
            elif self.use_swa:
                out.append("full" if i % self.swa_period == self.swa_period - 1 else "swa")
            else:
                out.append("full")
        return out

    def layer_window(self, i: int) -> int:
        """0 = full causal; >0 = sliding window of that many tokens incl. self."""
        return self.swa_window if self.layer_types()[i] == "swa" else 0

    def as_dict(self):
        return asdict(self)

    def replace(self, **kw) -> "Config":
        c = copy.deepcopy(self)
        names = {f.name for f in fields(Config)}
        for k, v in kw.items():
            if k not in names:
                raise KeyError(f"unknown config field {k!r}")
            setattr(c, k, v)
        return c


# ---------------------------------------------------------------------------
# Reference presets (config.py:166-314)
# ---------------------------------------------------------------------------
def smoke() -> Config:
    return Config(
        name="smoke", vocab_size=256, layers=2, d_model=64, n_q_heads=2,
        n_kv_heads=1, head_dim=32, n_experts=4, n_active=2, n_shared_experts=1,
        d_ff=128, dense_layers=1, batch_size=2, seq_len=128, train_steps=10,
        warmup_steps=2, learning_rate=1e-3, weight_decay=0.0, tokenizer="byte",
        log_every=1, mesh_data_axis=1, mesh_expert_axis=1,
        use_swa=True, swa_window=64, swa_period=2)


def smoke_kda() -> Config:
    c = smoke()
    c.name = "smoke_kda"
    c.use_swa = False
    c.use_kda = True
    c.kda_period = 2
    c.kda_heads = 2
    c.kda_head_dim = 32
    c.kda_chunk_size = 16
    c.use_scan = False
    return c


def full() -> Config:
    return Config(
        name="full", vocab_size=32000, layers=24, d_model=1536, n_q_heads=12,
        n_kv_heads=4, head_dim=128, n_experts=80, n_active=8, n_shared_experts=1,
        d_ff=768, dense_layers=3, batch_size=8, seq_len=16384,
        train_steps=100000, warmup_steps=2000, learning_rate=1e-4, min_lr=1e-5,
        decay_fraction=0.2, weight_decay=1.0, dtype="bf16", master_dtype="fp32",
        remat_policy="full", tokenizer="llama3", use_grain=True,
        mesh_data_axis=8, mesh_expert_axis=1, checkpoint_every=1000,
        log_every=10, infer_seq_len=32768, gen_every=1000)


def full_g4() -> Config:
    c = full()
    c.name = "full_g4"
    c.n_experts = 40
    c.n_active = 4
    c.d_ff = 1536
    c.d_ff_dense = 768
    return c


def custom() -> Config:
    c = full()
    c.name = "custom"
    c.dataset = "openbmb/Ultra-FineWeb-L3"
    c.dataset_files = ("hf://datasets/openbmb/Ultra-FineWeb-L3/"
                       "data/ultrafineweb_en_l3/multi_style/*.parquet")
    c.tokenizer = "llama3"
    c.vocab_size = 32000
    c.use_grain = True
    c.dataset_config = None
    return c


# ---------------------------------------------------------------------------
# Benchmark configurations (the BASELINE shapes)
# ---------------------------------------------------------------------------
def tiny_hybrid() -> Config:
    """Config 1: tiny hybrid MoE LM, fp32, CPU-runnable.

    4 layers [KDA, KDA, KDA, full]; d 256; 4 heads x 64 (GQA with 2 KV heads);
    KDA chunk 64 with per-channel sigmoid decay; 8 experts top-2 softmax router
    plus one shared expert, SwiGLU hidden 512; vocab 32768; batch 4 x 256;
    AdamW lr 3e-4 for 10 steps.
    """
    return Config(
        name="tiny_hybrid", vocab_size=32768, layers=4, d_model=256,
        n_q_heads=4, n_kv_heads=2, head_dim=64, n_experts=8, n_active=2,
        n_shared_experts=1, d_ff=512, dense_layers=0, batch_size=4, seq_len=256,
        train_steps=10, learning_rate=3e-4, min_lr=3e-4, warmup_steps=0,
        decay_fraction=0.0, weight_decay=0.1, dtype="fp32", use_kda=True,
        kda_period=4, kda_heads=4, kda_head_dim=64, kda_chunk_size=64,
        use_scan=False, optimizer="adamw", router_type="softmax",
        aux_loss_weight=0.01, kda_gate="sigmoid", tokenizer="byte",
        infer_seq_len=256, remat=False)


def hybrid_1p3b() -> Config:
    """Config 2 (flagship): hybrid MoE ~1.3B total, bf16, FSDP over the box.

    16 layers, 3:1 KDA:full; d 1024; 16 heads x 64 (full attention uses 4 KV
    heads); 32 experts top-4 plus one shared expert; SwiGLU hidden 768; router
    balance loss 0.01; vocab 32768; seq 4096 x global batch 256; AdamW with
    bf16 working weights and fp32 master weights.
    """
    return Config(
        name="hybrid_1p3b", vocab_size=32768, layers=16, d_model=1024,
        n_q_heads=16, n_kv_heads=4, head_dim=64, n_experts=32, n_active=4,
        n_shared_experts=1, d_ff=768, dense_layers=0, batch_size=256,
        seq_len=4096, train_steps=1000, learning_rate=3e-4, min_lr=3e-5,
        warmup_steps=100, decay_fraction=0.2, weight_decay=0.1, dtype="bf16",
        use_kda=True, kda_period=4, kda_heads=16, kda_head_dim=64,
        kda_chunk_size=64, use_scan=False, optimizer="adamw",
        balance_loss_weight=0.01, tokenizer="byte", mesh_data_axis=8,
        infer_seq_len=4096, remat=False, micro_batch=8)


def ep_moe() -> Config:
    """Config 3: expert-parallel MoE, EP=8; 24 layers 3:1 KDA:full; d 2048;
    16 heads x 128 (4 KV heads); 64 experts (8 per GPU) top-8 + shared; SwiGLU
    hidden 1408; capacity factor 1.25; seq 4096 x global batch 512."""
    return Config(
        name="ep_moe", vocab_size=32768, layers=24, d_model=2048, n_q_heads=16,
        n_kv_heads=4, head_dim=128, n_experts=64, n_active=8, n_shared_experts=1,
        d_ff=1408, dense_layers=0, batch_size=512, seq_len=4096,
        train_steps=1000, learning_rate=3e-4, min_lr=3e-5, warmup_steps=100,
        weight_decay=0.1, use_kda=True, kda_period=4, kda_heads=16,
        kda_head_dim=128, use_scan=False, optimizer="adamw",
        balance_loss_weight=0.01, capacity_factor=1.25, mesh_data_axis=1,
        mesh_expert_axis=8, infer_seq_len=4096, remat=False, micro_batch=4)


def long_kda() -> Config:
    """Config 4: the 1.3B hybrid at seq 32768 x global batch 16."""
    c = hybrid_1p3b()
    c.name = "long_kda"
    c.seq_len = 32768
    c.batch_size = 16
    c.infer_seq_len = 32768
    c.micro_batch = 1
    return c


PRESETS = {"smoke": smoke, "smoke_kda": smoke_kda, "full": full,
           "full_g4": full_g4, "custom": custom, "tiny_hybrid": tiny_hybrid,
           "hybrid_1p3b": hybrid_1p3b, "ep_moe": ep_moe, "long_kda": long_kda}


def get_config(name: str) -> Config:
    if name not in PRESETS:
        raise ValueError(f"Unknown config preset: {name!r}. Choose from {list(PRESETS)}")
    return PRESETS[name]()
