"""Typed training configuration and its YAML loader.

The schema keeps every key of the reference's YAML files so the same files
drive ``train.py`` here (reference: ``src/config.py:44-215`` for the sections,
``src/config.py:219-326`` for the top level).  Two additions:

* ``kernels:`` — an optional section holding switches for the native fast
  paths (fused collectives).  Files without it parse unchanged.
* ``data.dataset_path: uniform`` — uniform-random token ids, the synthetic
  workload used by the throughput benchmarks.

Loading rules (same contract as ``src/config.py:329-356``): nested dicts become
nested dataclasses, YAML lists become tuples where the field is a tuple, and an
unknown key raises ``TypeError`` naming the valid keys, on every rank, before
any process group exists.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field, fields, is_dataclass
from typing import Any

import yaml

VALID_SHARDING = ("FULL_SHARD", "HYBRID_SHARD", "SHARD_GRAD_OP", "NO_SHARD")
VALID_PREFETCH = ("BACKWARD_PRE", "BACKWARD_POST")


@dataclass
class ModelConfig:
    """LLaMA-style decoder hyper-parameters (reference ``src/config.py:44-114``).

    ``n_kv_heads`` defaults to ``n_heads`` (plain multi-head attention) and
    ``ffn_hidden_size`` defaults to ``8/3 * d_model`` rounded up to a multiple
    of 256, the LLaMA SwiGLU sizing.
    """

    vocab_size: int = 32000
    d_model: int = 768
    n_layers: int = 12
    n_heads: int = 12
    n_kv_heads: int | None = None
    ffn_hidden_size: int | None = None
    max_seq_len: int = 2048
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    tie_embeddings: bool = True
    dropout: float = 0.0
    attention_bias: bool = False
    mlp_bias: bool = False

    def __post_init__(self) -> None:
        if self.n_kv_heads is None:
            self.n_kv_heads = self.n_heads
        if self.ffn_hidden_size is None:
            raw = int(8 * self.d_model / 3)
            self.ffn_hidden_size = -(-raw // 256) * 256

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def kv_dim(self) -> int:
        assert self.n_kv_heads is not None
        return self.n_kv_heads * self.head_dim

    def num_parameters(self) -> int:
        """Analytic parameter count used by MFU: embedding, blocks, untied head.

        Norm weights and biases are left out, as in ``src/config.py:97-114``.
        """
        assert self.ffn_hidden_size is not None
        d = self.d_model
        attn = 2 * d * d + 2 * d * self.kv_dim
        mlp = 3 * d * self.ffn_hidden_size
        head = 0 if self.tie_embeddings else self.vocab_size * d
        return self.vocab_size * d + self.n_layers * (attn + mlp) + head


@dataclass
class ParallelConfig:
    """2D mesh and sharding policy (reference ``src/config.py:118-154``).

    ``dp_size == -1`` means "infer as world_size // tp_size".
    ``sharding_strategy``: FULL_SHARD (params, grads and optimizer state
    sharded; params re-gathered for backward), SHARD_GRAD_OP (params stay
    gathered between forward and backward), NO_SHARD (replicated, grads
    all-reduced), HYBRID_SHARD (shard inside a node, replicate across nodes;
    on a single node it is FULL_SHARD).
    ``cpu_offload`` is accepted for YAML compatibility; the engine keeps all
    state in HBM (it is never read by the reference either).
    ``param_dtype`` is the compute and gathered-parameter dtype.  Gradients
    are always accumulated and reduced in float32 and the RoPE tables are
    float32 whatever ``reduce_dtype`` / ``buffer_dtype`` say (a warning is
    issued when ``reduce_dtype`` asks for less).
    """

    tp_size: int = 1
    dp_size: int = -1
    sharding_strategy: str = "FULL_SHARD"
    activation_checkpointing: bool = False
    sequence_parallel: bool = False
    backward_prefetch: str = "BACKWARD_PRE"
    forward_prefetch: bool = True
    limit_all_gathers: bool = True
    cpu_offload: bool = False
    param_dtype: str = "bfloat16"
    reduce_dtype: str = "float32"
    buffer_dtype: str = "bfloat16"
    loss_parallel: bool = False


@dataclass
class OptimizerConfig:
    """AdamW / LAMB hyper-parameters (reference ``src/config.py:158-176``).

    ``decay_flat_params_under_fsdp``: the reference builds its decay groups
    after FSDP flattening, so every parameter is 1-D and no decay is applied
    under FSDP.  ``False`` (default) applies decay to every >=2-D weight as the
    reference documents; ``True`` reproduces the reference's runtime behaviour
    for loss-parity runs.
    """

    name: str = "adamw"
    lr: float = 3e-4
    weight_decay: float = 0.1
    betas: tuple[float, float] = (0.9, 0.95)
    eps: float = 1e-8
    fused: bool = True
    decay_flat_params_under_fsdp: bool = False


@dataclass
class SchedulerConfig:
    """Linear warmup then cosine decay to ``min_lr`` (``src/config.py:180-191``)."""

    warmup_steps: int = 100
    max_steps: int = 10000
    min_lr: float = 3e-5


@dataclass
class DataConfig:
    """Data pipeline (reference ``src/config.py:195-215``).

    ``dataset_path``: ``synthetic`` (learnable Markov tokens), ``uniform``
    (uniform-random ids) or a path to a uint16 ``.bin`` token file.
    """

    dataset_path: str = "synthetic"
    tokenizer_name: str = "gpt2"
    seq_len: int = 1024
    micro_batch_size: int = 8
    global_batch_size: int = 64
    num_workers: int = 2
    shuffle: bool = True


@dataclass
class KernelConfig:
    """Switches for the native fast paths (no reference counterpart).

    ``fused_comm``: TP/DP collectives run as this package's peer-memory kernels
    (``False`` routes them through ``torch.distributed``/NCCL, the baseline).
    ``deterministic``: fixed-order reductions everywhere (bit-exact reruns).
    """

    fused_comm: bool = True
    deterministic: bool = True


@dataclass
class TrainingConfig:
    """Top-level config (reference ``src/config.py:219-326``)."""

    model: ModelConfig = field(default_factory=ModelConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    data: DataConfig = field(default_factory=DataConfig)
    kernels: KernelConfig = field(default_factory=KernelConfig)

    seed: int = 1234
    grad_accum_steps: int = 1
    max_grad_norm: float = 1.0
    max_steps: int = 10000
    log_interval: int = 10
    eval_interval: int = 500
    eval_steps: int = 20
    save_interval: int = 1000
    warmup_profile_steps: int = 5
    profile_steps: int = 3
    checkpoint_dir: str = "checkpoints"
    run_id: str = "run"
    resume_from: str | None = None
    backend: str = "nccl"

    def validate(self, world_size: int, dp_size: int, tp_size: int | None = None) -> None:
        """Cross-field checks that need the runtime topology.

        Same checks as ``src/config.py:259-294`` (global-batch identity with
        auto-derivation when ``global_batch_size <= 0``, ``d_model % n_heads``,
        strategy names) plus the head/TP divisibility checks the reference
        lacks (a tp that does not divide ``n_kv_heads`` crashed inside
        attention there).
        """
        want = self.data.micro_batch_size * self.grad_accum_steps * dp_size
        if self.data.global_batch_size <= 0:
            self.data.global_batch_size = want
        elif self.data.global_batch_size != want:
            raise ValueError(
                f"global_batch_size={self.data.global_batch_size} does not equal "
                f"micro_batch_size({self.data.micro_batch_size}) x grad_accum_steps"
                f"({self.grad_accum_steps}) x dp_size({dp_size}) = {want}; change "
                "one of them."
            )
        m = self.model
        if m.d_model % m.n_heads:
            raise ValueError(f"d_model={m.d_model} is not a multiple of n_heads={m.n_heads}.")
        if self.parallel.sharding_strategy not in VALID_SHARDING:
            raise ValueError(
                f"sharding_strategy={self.parallel.sharding_strategy!r} is not one of "
                f"{sorted(VALID_SHARDING)}."
            )
        if self.parallel.backward_prefetch not in VALID_PREFETCH:
            raise ValueError(
                f"backward_prefetch={self.parallel.backward_prefetch!r} is not one of "
                f"{sorted(VALID_PREFETCH)}."
            )
        tp = tp_size if tp_size is not None else world_size // max(dp_size, 1)
        assert m.n_kv_heads is not None and m.ffn_hidden_size is not None
        for name, value in (("n_heads", m.n_heads), ("n_kv_heads", m.n_kv_heads),
                            ("ffn_hidden_size", m.ffn_hidden_size)):
            if value % tp:
                raise ValueError(f"{name}={value} is not divisible by tp_size={tp}.")
        if m.n_heads % m.n_kv_heads:
            raise ValueError(f"n_heads={m.n_heads} is not a multiple of n_kv_heads={m.n_kv_heads}.")
        if self.parallel.loss_parallel and m.vocab_size % tp:
            raise ValueError(f"loss_parallel needs vocab_size={m.vocab_size} divisible by tp={tp}.")
        if self.parallel.sequence_parallel and tp > 1:
            tokens = self.data.micro_batch_size * self.data.seq_len
            if tokens % tp:
                raise ValueError(
                    f"sequence_parallel needs micro_batch_size*seq_len={tokens} divisible by tp={tp}."
                )

    @classmethod
    def from_yaml(cls, path: str) -> TrainingConfig:
        with open(path) as f:
            raw = yaml.safe_load(f) or {}
        return cls.from_dict(raw)

    @classmethod
    def from_dict(cls, raw: dict[str, Any]) -> TrainingConfig:
        return _build(cls, raw)

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)


def _build(cls: type, raw: dict[str, Any]) -> Any:
    """Instantiate dataclass ``cls`` from ``raw``, recursing into sub-configs."""
    by_name = {f.name: f for f in fields(cls)}
    kwargs: dict[str, Any] = {}
    for key, value in raw.items():
        if key not in by_name:
            raise TypeError(
                f"Unknown config key {key!r} for {cls.__name__}; valid keys: {sorted(by_name)}."
            )
        f = by_name[key]
        sub = _nested_type(f)
        if sub is not None and isinstance(value, dict):
            kwargs[key] = _build(sub, value)
        elif isinstance(value, list) and "tuple" in str(f.type):
            kwargs[key] = tuple(value)
        else:
            kwargs[key] = value
    return cls(**kwargs)


def _nested_type(f: dataclasses.Field) -> type | None:
    factory = f.default_factory  # type: ignore[misc]
    if factory is dataclasses.MISSING:
        return None
    probe = factory()
    return type(probe) if is_dataclass(probe) else None
