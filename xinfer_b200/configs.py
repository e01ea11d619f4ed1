"""Model geometries of the Qwen3 / Qwen3.5 families served by the decode megakernel.

Field meaning follows the HF configs the reference loads (compiler/qwen3/model.py:16-26,
compiler/qwen35/model.py:21-42); the benchmark geometries are the ones BASELINE names
(Qwen3-0.6B, Qwen3.5-0.8B, Qwen3.5-4B). The reference adapters pin the head geometry: Qwen3
attention 16/8 x 128 (compiler/qwen3/adapters/attention.py:18-23); DeltaNet 16 key heads,
16 or 32 value heads, K = V = 128, width-4 SiLU conv (compiler/qwen35/adapters/delta.py:17-31).
The small "tiny" configs keep that head geometry and shrink hidden size, depth and vocabulary
so the CPU oracle and the reference's own code finish in seconds.
"""

from dataclasses import dataclass, field, replace

QWEN3 = "qwen3"
QWEN35 = "qwen3.5"


@dataclass(frozen=True)
class Geometry:
    name: str
    family: str
    num_layers: int
    hidden: int
    intermediate: int
    vocab: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float
    partial_rotary_factor: float = 1.0
    rms_eps: float = 1e-6
    lin_key_heads: int = 0
    lin_value_heads: int = 0
    lin_head_dim: int = 128
    conv_width: int = 4
    full_attention_interval: int = 4
    max_position_embeddings: int = 32768
    layer_types: tuple = field(default=())

    def __post_init__(self):
        if not self.layer_types:
            if self.family == QWEN35:
                kinds = tuple(
                    "linear_attention" if (i + 1) % self.full_attention_interval else "full_attention"
                    for i in range(self.num_layers)
                )
            else:
                kinds = ("full_attention",) * self.num_layers
            object.__setattr__(self, "layer_types", kinds)

    @property
    def rotary_dim(self):
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def conv_channels(self):
        return (2 * self.lin_key_heads + self.lin_value_heads) * self.lin_head_dim

    @property
    def q_rows(self):
        """q_proj output rows: Qwen3.5 interleaves [query | gate] per head."""
        return self.num_q_heads * self.head_dim * (2 if self.family == QWEN35 else 1)

    def is_delta(self, layer):
        return self.layer_types[layer] == "linear_attention"


QWEN3_0_6B = Geometry(
    name="qwen3-0.6b", family=QWEN3, num_layers=28, hidden=1024, intermediate=3072,
    vocab=151936, num_q_heads=16, num_kv_heads=8, head_dim=128, rope_theta=1e6,
    max_position_embeddings=40960,
)
QWEN35_0_8B = Geometry(
    name="qwen3.5-0.8b", family=QWEN35, num_layers=24, hidden=1024, intermediate=3584,
    vocab=248320, num_q_heads=8, num_kv_heads=2, head_dim=256, rope_theta=10000.0,
    partial_rotary_factor=0.25, lin_key_heads=16, lin_value_heads=16,
    max_position_embeddings=262144,
)
QWEN35_4B = Geometry(
    name="qwen3.5-4b", family=QWEN35, num_layers=32, hidden=2560, intermediate=9216,
    vocab=248320, num_q_heads=16, num_kv_heads=4, head_dim=256, rope_theta=10000.0,
    partial_rotary_factor=0.25, lin_key_heads=16, lin_value_heads=32,
    max_position_embeddings=262144,
)
QWEN3_TINY = replace(
    QWEN3_0_6B, name="qwen3-tiny", num_layers=2, hidden=256, intermediate=512, vocab=1024,
    layer_types=(),
)
QWEN35_TINY = replace(
    QWEN35_0_8B, name="qwen3.5-tiny", num_layers=4, hidden=256, intermediate=512, vocab=1024,
    layer_types=(),
)
QWEN35_TINY_HV32 = replace(
    QWEN35_4B, name="qwen3.5-tiny-hv32", num_layers=4, hidden=256, intermediate=768, vocab=1280,
    layer_types=(),
)

# Full-width, reduced-depth variants: every kernel runs at its real dimensions (hidden, heads,
# vocabulary) while the shallow stack keeps one-ulp rounding flips from cascading, so parity can
# be held to the tight bar at full width.
QWEN3_0_6B_L2 = replace(QWEN3_0_6B, name="qwen3-0.6b-l2", num_layers=2, layer_types=())
QWEN35_0_8B_L4 = replace(QWEN35_0_8B, name="qwen3.5-0.8b-l4", num_layers=4, layer_types=())
QWEN35_4B_L4 = replace(QWEN35_4B, name="qwen3.5-4b-l4", num_layers=4, layer_types=())

# The smallest geometry the kernels take (one DeltaNet and one attention layer, one key / two
# value DeltaNet heads): for format tests whose fixtures are committed (a bundle archive).
QWEN35_MICRO = replace(
    QWEN35_0_8B, name="qwen3.5-micro", num_layers=2, hidden=256, intermediate=64, vocab=128,
    num_q_heads=2, num_kv_heads=1, lin_key_heads=1, lin_value_heads=2, full_attention_interval=2,
    layer_types=(),
)

CONFIGS = {
    g.name: g
    for g in (QWEN3_0_6B, QWEN35_0_8B, QWEN35_4B, QWEN3_TINY, QWEN35_TINY, QWEN35_TINY_HV32,
              QWEN3_0_6B_L2, QWEN35_0_8B_L4, QWEN35_4B_L4, QWEN35_MICRO)
}


def get(name):
    try:
        return CONFIGS[name]
    except KeyError:
        raise ValueError(f"unknown model config {name!r}; known: {sorted(CONFIGS)}") from None


def hf_config(geometry):
    """The transformers config object for a geometry (used by tests and the CPU baseline)."""
    if geometry.family == QWEN3:
        from transformers import Qwen3Config

        return Qwen3Config(
            vocab_size=geometry.vocab, hidden_size=geometry.hidden,
            intermediate_size=geometry.intermediate, num_hidden_layers=geometry.num_layers,
            num_attention_heads=geometry.num_q_heads, num_key_value_heads=geometry.num_kv_heads,
            head_dim=geometry.head_dim, rms_norm_eps=geometry.rms_eps,
            rope_parameters={"rope_type": "default", "rope_theta": geometry.rope_theta},
            tie_word_embeddings=True, max_position_embeddings=geometry.max_position_embeddings,
            attention_bias=False,
        )
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextConfig

    return Qwen3_5TextConfig(
        vocab_size=geometry.vocab, hidden_size=geometry.hidden,
        intermediate_size=geometry.intermediate, num_hidden_layers=geometry.num_layers,
        num_attention_heads=geometry.num_q_heads, num_key_value_heads=geometry.num_kv_heads,
        head_dim=geometry.head_dim, rms_norm_eps=geometry.rms_eps,
        rope_parameters={
            "rope_type": "default", "rope_theta": geometry.rope_theta,
            "partial_rotary_factor": geometry.partial_rotary_factor,
        },
        linear_num_key_heads=geometry.lin_key_heads, linear_num_value_heads=geometry.lin_value_heads,
        linear_key_head_dim=geometry.lin_head_dim, linear_value_head_dim=geometry.lin_head_dim,
        linear_conv_kernel_dim=geometry.conv_width, tie_word_embeddings=True,
        max_position_embeddings=geometry.max_position_embeddings,
        layer_types=list(geometry.layer_types),
    )
