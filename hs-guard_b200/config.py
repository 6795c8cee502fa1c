"""Architecture constants of the HS-Guard streaming classifier.

The backbone is the Qwen3.5-0.8B hybrid: 24 layers, every fourth one a gated softmax-attention layer
restricted to a 512-token window, the rest gated-delta-rule ("GDN") linear-attention layers
(reference: ``docs/technical_report.tex:30``; layer pattern from transformers
``Qwen3_5TextConfig.__post_init__`` with ``full_attention_interval=4``). Two role heads
(``user``, ``assistant``) read the final hidden state: Linear(1024->512) -> LayerNorm -> SiLU ->
Linear(512->3) (reference ``src/hs_guard/runtime.py:54-75``). With these shapes the model has
754,519,918 parameters, the published count.

The CUDA kernels are specialised to exactly these sizes; ``HsgConfig.check`` rejects anything else.
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict

LABELS = ("safe", "unsafe", "controversial")
ROLES = ("user", "assistant")
# Session-row buckets of StreamingGuard (reference runtime.py:154) and token buckets of a tick
# (reference engine/bucketed_engine.py:9).
SESSION_BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 352, 384, 448, 512)
TOKEN_BUCKETS = (1, 2, 4, 8, 16, 32, 64)


@dataclass(frozen=True)
class HsgConfig:
    hidden: int = 1024
    intermediate: int = 3584
    n_layers: int = 24
    full_attn_interval: int = 4
    gdn_heads: int = 16            # key heads == value heads
    gdn_head_dim: int = 128        # dk == dv
    conv_kernel: int = 4
    attn_heads: int = 8
    kv_heads: int = 2
    attn_head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10000.0    # not shape-affecting; transformers' default, pinned here
    rms_eps: float = 1e-6
    head_ln_eps: float = 1e-5
    vocab: int = 248320
    window: int = 512
    head_hidden: int = 512
    n_classes: int = 3
    roles: tuple = field(default=ROLES)

    # ---- derived sizes -------------------------------------------------------------------
    @property
    def layer_types(self):
        return ["full_attention" if (i + 1) % self.full_attn_interval == 0 else "linear_attention"
                for i in range(self.n_layers)]

    @property
    def n_gdn(self):
        return self.layer_types.count("linear_attention")

    @property
    def n_attn(self):
        return self.layer_types.count("full_attention")

    @property
    def key_dim(self):
        return self.gdn_heads * self.gdn_head_dim

    @property
    def conv_dim(self):
        return 3 * self.key_dim

    @property
    def gdn_in_rows(self):
        """Rows of the fused GDN input projection: qkv | z | b | a, padded to a multiple of 128."""
        rows = self.conv_dim + self.key_dim + 2 * self.gdn_heads
        return (rows + 127) // 128 * 128

    @property
    def attn_in_rows(self):
        """Rows of the fused attention input projection: q(+gate) | k | v."""
        return 2 * self.attn_heads * self.attn_head_dim + 2 * self.kv_heads * self.attn_head_dim

    @property
    def rotary_dim(self):
        return int(self.attn_head_dim * self.partial_rotary_factor)

    def layer_index(self):
        """[(kind, index within kind)] per layer, as reference engine/bucketed_engine.py:31."""
        types = self.layer_types
        return [(t, sum(1 for u in types[:i] if u == t)) for i, t in enumerate(types)]

    def hf_kwargs(self):
        """Keyword arguments for transformers' Qwen3_5TextConfig describing the same backbone."""
        return dict(hidden_size=self.hidden, intermediate_size=self.intermediate, num_hidden_layers=self.n_layers,
                    num_attention_heads=self.attn_heads, num_key_value_heads=self.kv_heads,
                    head_dim=self.attn_head_dim, linear_num_key_heads=self.gdn_heads,
                    linear_num_value_heads=self.gdn_heads, linear_key_head_dim=self.gdn_head_dim,
                    linear_value_head_dim=self.gdn_head_dim, linear_conv_kernel_dim=self.conv_kernel,
                    vocab_size=self.vocab, rms_norm_eps=self.rms_eps,
                    rope_parameters={"rope_type": "default", "rope_theta": self.rope_theta,
                                     "partial_rotary_factor": self.partial_rotary_factor})

    def check(self):
        """Raise ValueError unless this is the architecture the kernels are built for."""
        if self != HsgConfig(rope_theta=self.rope_theta, rms_eps=self.rms_eps, head_ln_eps=self.head_ln_eps,
                             vocab=self.vocab, window=self.window):
            raise ValueError(f"unsupported architecture: {asdict(self)}")
        if self.window != 512:
            raise ValueError("the ring kernels are built for a 512-token window")
        return self

    @classmethod
    def from_hf(cls, hf_config, window=512):
        """Read the shape-relevant fields of a transformers Qwen3_5TextConfig."""
        rope = getattr(hf_config, "rope_parameters", None) or {}
        types = list(hf_config.layer_types[:hf_config.num_hidden_layers])
        interval = types.index("full_attention") + 1 if "full_attention" in types else 0
        cfg = cls(hidden=hf_config.hidden_size, intermediate=hf_config.intermediate_size,
                  n_layers=hf_config.num_hidden_layers, full_attn_interval=interval,
                  gdn_heads=hf_config.linear_num_value_heads, gdn_head_dim=hf_config.linear_value_head_dim,
                  conv_kernel=hf_config.linear_conv_kernel_dim, attn_heads=hf_config.num_attention_heads,
                  kv_heads=hf_config.num_key_value_heads, attn_head_dim=hf_config.head_dim,
                  partial_rotary_factor=rope.get("partial_rotary_factor", 0.25),
                  rope_theta=float(rope.get("rope_theta", 10000.0)), rms_eps=hf_config.rms_norm_eps,
                  vocab=hf_config.vocab_size, window=window)
        if types != cfg.layer_types or hf_config.linear_num_key_heads != cfg.gdn_heads \
                or hf_config.linear_key_head_dim != cfg.gdn_head_dim:
            raise ValueError("unsupported layer pattern or GDN head layout")
        return cfg


DEFAULT = HsgConfig()
