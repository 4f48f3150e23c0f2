"""Qwen3 decoder shapes and the synthetic (seeded) weight recipe.

The reference pins one shape, Qwen3-8B (qwen3/model.hpp:11-22); this build is
shape-generic and names the configurations it is measured on. Weights of a
synthetic model are drawn per tensor from a seeded counter-based generator
(the same bits on the GPU, in libxpu_cuda's xpu_fill_normal_bf16, and on the
CPU), so a model is fully described by (shape, seed) and never written to disk.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

HEAD_DIM = 128
ROPE_THETA = 1_000_000.0
RMS_EPS = 1e-6
EOS_TOKEN = 151645          # qwen3/model.hpp:19
END_OF_TURN_TOKEN = 151643  # qwen3/model.hpp:20
MAX_CONTEXT = 40960         # qwen3/model.hpp:18
WEIGHT_STD = 0.02

# Per-layer tensor suffixes in the canonical order used for seeding and for
# the C oracle's tensor table (qwen3/model.cpp:415-420 lists the same names).
LAYER_TENSORS = (
    "input_layernorm.weight", "post_attention_layernorm.weight",
    "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
    "self_attn.o_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
    "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight",
)


@dataclass(frozen=True)
class Qwen3Shape:
    hidden: int
    intermediate: int
    layers: int
    q_heads: int
    kv_heads: int
    vocab: int
    tied: bool
    eps: float = RMS_EPS
    rope_theta: float = ROPE_THETA

    def as_dict(self) -> dict:
        return asdict(self)

    def tensor_names(self) -> list[str]:
        names = ["model.embed_tokens.weight", "model.norm.weight"]
        if not self.tied:
            names.append("lm_head.weight")
        for layer in range(self.layers):
            names += [f"model.layers.{layer}.{s}" for s in LAYER_TENSORS]
        return names

    def shape_of(self, name: str) -> tuple[int, ...]:
        H, I, V = self.hidden, self.intermediate, self.vocab
        q, kv = self.q_heads * HEAD_DIM, self.kv_heads * HEAD_DIM
        if name in ("model.embed_tokens.weight", "lm_head.weight"):
            return (V, H)
        if name == "model.norm.weight":
            return (H,)
        suffix = name.split(".", 3)[3]
        return {
            "input_layernorm.weight": (H,), "post_attention_layernorm.weight": (H,),
            "self_attn.q_proj.weight": (q, H), "self_attn.k_proj.weight": (kv, H),
            "self_attn.v_proj.weight": (kv, H), "self_attn.o_proj.weight": (H, q),
            "self_attn.q_norm.weight": (HEAD_DIM,), "self_attn.k_norm.weight": (HEAD_DIM,),
            "mlp.gate_proj.weight": (I, H), "mlp.up_proj.weight": (I, H),
            "mlp.down_proj.weight": (H, I),
        }[suffix]

    def tensor_tag(self, name: str) -> int:
        """Generator stream of a tensor: 0 embed, 1 final norm, 2 lm_head,
        3 + 11*layer + position in LAYER_TENSORS."""
        if name == "model.embed_tokens.weight":
            return 0
        if name == "model.norm.weight":
            return 1
        if name == "lm_head.weight":
            return 2
        _, _, layer, suffix = name.split(".", 3)
        return 3 + 11 * int(layer) + LAYER_TENSORS.index(suffix)

    @staticmethod
    def is_norm(name: str) -> bool:
        return name.endswith("norm.weight")

    def weight_bytes(self) -> int:
        return sum(2 * _prod(self.shape_of(n)) for n in self.tensor_names())

    def streamed_bytes_per_token(self) -> int:
        """Weight bytes one decode step reads: every tensor once, except the
        embedding table, of which only one row is read (the lm_head, tied or
        not, is read whole)."""
        total = self.weight_bytes() - 2 * self.vocab * self.hidden + 2 * self.hidden
        if self.tied:
            total += 2 * self.vocab * self.hidden
        return total

    def kv_bytes_per_position(self) -> int:
        return self.layers * 2 * self.kv_heads * HEAD_DIM * 2


def _prod(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


PRESETS: dict[str, Qwen3Shape] = {
    # 28 layers, hidden 1024, 16/8 heads, I 3072, tied.
    "qwen3-0.6b": Qwen3Shape(hidden=1024, intermediate=3072, layers=28, q_heads=16, kv_heads=8,
                             vocab=151936, tied=True),
    # 36 layers, hidden 4096, 32/8 heads, I 12288, untied.
    "qwen3-8b": Qwen3Shape(hidden=4096, intermediate=12288, layers=36, q_heads=32, kv_heads=8,
                           vocab=151936, tied=False),
    # Qwen3-8B layer and vocabulary shapes, two layers: the 8B kernels' tiling
    # (split-K QKV, 8 x 512 / 8 x 1536 canonical chunks) at CPU-checkable cost.
    "qwen3-8b-l2": Qwen3Shape(hidden=4096, intermediate=12288, layers=2, q_heads=32, kv_heads=8,
                              vocab=151936, tied=False),
    # Small shapes for CPU-checked parity tests.
    "tiny": Qwen3Shape(hidden=256, intermediate=768, layers=2, q_heads=4, kv_heads=2,
                       vocab=4096, tied=False),
    "tiny-tied": Qwen3Shape(hidden=512, intermediate=1024, layers=3, q_heads=8, kv_heads=2,
                            vocab=3072, tied=True),
}
