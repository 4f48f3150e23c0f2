"""Qwen3 model oracles (test infrastructure only).

Two CPU implementations of one greedy decode step, used as checkers and as
the timed CPU baseline:

* ``CDecoder``: oracle/xpu_oracle.c ``orc_qwen3_decode``, a C restatement of
  the transformers eager/bf16 forward with its rounding points (token-by-token,
  KV cache, FP32 accumulation).
* ``HFDecoder``: the reference's own model oracle, qwen3/reference.py:11-45,
  restated: a transformers ``Qwen3ForCausalLM`` in bf16 with
  ``attn_implementation="eager"``, here built from a config plus seeded
  weights instead of ``from_pretrained`` (no checkpoint is available). The
  modelling code is third-party: transformers (reference pins 4.51.0 in
  qwen3/requirements.txt:2; this image has the version ``hf_version()``
  returns, recorded with every fixture).

Weights come from ``seeded_weights`` - the generator that libxpu_cuda's
``xpu_fill_normal_bf16`` reproduces bit for bit on the GPU.
"""

from __future__ import annotations

import ctypes

import numpy as np

from xpu_playground_b200.qwen3_config import HEAD_DIM, WEIGHT_STD, Qwen3Shape

from . import oracle as orc

BF16_ONE = 0x3F80


def seeded_weights(shape: Qwen3Shape, seed: int) -> dict[str, np.ndarray]:
    """name -> bf16 bit array. Norm weights are 1 (the transformers init);
    every other tensor is N(0, 0.02) from stream ``shape.tensor_tag(name)``."""
    out = {}
    for name in shape.tensor_names():
        dims = shape.shape_of(name)
        n = int(np.prod(dims))
        if shape.is_norm(name):
            out[name] = np.full(dims, BF16_ONE, np.uint16)
        else:
            out[name] = orc.normal_bf16(n, seed, shape.tensor_tag(name), WEIGHT_STD).reshape(dims)
    return out


def prompt_ids(n: int, vocab: int, seed: int) -> list[int]:
    """Seeded uniform token ids in [0, vocab)."""
    rng = np.random.default_rng(seed)
    return [int(t) for t in rng.integers(0, vocab, size=n)]


class CDecoder:
    """Token-by-token greedy decoding with the C restatement."""

    def __init__(self, shape: Qwen3Shape, weights: dict[str, np.ndarray], max_seq: int):
        self.shape, self.max_seq = shape, max_seq
        names = ["model.embed_tokens.weight", "model.norm.weight",
                 "model.embed_tokens.weight" if shape.tied else "lm_head.weight"]
        for layer in range(shape.layers):
            names += [f"model.layers.{layer}.{s}" for s in
                      ("input_layernorm.weight", "post_attention_layernorm.weight",
                       "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                       "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                       "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                       "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")]
        self._keep = [np.ascontiguousarray(weights[n]) for n in names]
        self._table = (ctypes.c_void_p * len(names))(*[a.ctypes.data for a in self._keep])
        kv = shape.layers * max_seq * shape.kv_heads * HEAD_DIM
        self.kc = np.zeros(kv, np.uint16)
        self.vc = np.zeros(kv, np.uint16)
        self.cos, self.sin = orc.rope_tables(max_seq, shape.rope_theta)
        self.cfg = orc.Qwen3Config(shape.hidden, shape.intermediate, shape.q_heads, shape.kv_heads,
                                   shape.layers, shape.vocab, max_seq, shape.eps)

    def step(self, token: int, position: int, want_logits: bool = True):
        logits = np.empty(self.shape.vocab, np.uint16) if want_logits else None
        nxt = orc.lib().orc_qwen3_decode(ctypes.byref(self.cfg), self._table, self.kc, self.vc,
                                         self.cos, self.sin, token, position,
                                         logits.ctypes.data if want_logits else None)
        return int(nxt), logits


def hf_version() -> str:
    import transformers
    return transformers.__version__


class HFDecoder:
    """qwen3/reference.py's model, built from (shape, weights)."""

    def __init__(self, shape: Qwen3Shape, weights: dict[str, np.ndarray], threads: int | None = None):
        import torch
        from transformers import Qwen3Config, Qwen3ForCausalLM

        if threads:
            torch.set_num_threads(threads)
        self.torch = torch
        cfg = Qwen3Config(
            hidden_size=shape.hidden, intermediate_size=shape.intermediate,
            num_hidden_layers=shape.layers, num_attention_heads=shape.q_heads,
            num_key_value_heads=shape.kv_heads, head_dim=HEAD_DIM, vocab_size=shape.vocab,
            tie_word_embeddings=shape.tied, rms_norm_eps=shape.eps,
            rope_theta=shape.rope_theta, max_position_embeddings=40960,
            attn_implementation="eager", torch_dtype="bfloat16")
        with torch.device("meta"):
            model = Qwen3ForCausalLM(cfg)
        model = model.to_empty(device="cpu").to(torch.bfloat16)
        state = {}
        for name, bits in weights.items():
            t = torch.from_numpy(bits.astype(np.int16).view(np.int16)).view(torch.bfloat16)
            state[name] = t.reshape(shape.shape_of(name))
        missing, unexpected = model.load_state_dict(state, strict=False, assign=True)
        missing = [m for m in missing if not (shape.tied and m == "lm_head.weight")]
        if missing or unexpected:
            raise RuntimeError(f"state dict mismatch: missing={missing} unexpected={unexpected}")
        if shape.tied:
            model.tie_weights()
        # Buffers created on the meta device carry no values: rebuild the
        # rotary embedding (its inv_freq) on the CPU.
        from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
        model.model.rotary_emb = Qwen3RotaryEmbedding(config=cfg)
        self.model = model.eval()
        self.past = None

    def step(self, token: int, position: int):
        """One cached forward of one token; returns (argmax id, bf16 logit bits)."""
        torch = self.torch
        with torch.no_grad():
            out = self.model(input_ids=torch.tensor([[token]]),
                             position_ids=torch.tensor([[position]]),
                             past_key_values=self.past, use_cache=True, return_dict=True)
        self.past = out.past_key_values
        logits = out.logits[0, -1]
        bits = logits.view(torch.int16).numpy().view(np.uint16).copy()
        return int(torch.argmax(logits.float()).item()), bits

    def generate(self, ids: list[int], max_new_tokens: int) -> list[int]:
        """reference.py:38-44: greedy generate with batched prefill."""
        torch = self.torch
        with torch.no_grad():
            out = self.model.generate(torch.tensor([ids]), max_new_tokens=max_new_tokens,
                                      do_sample=False, use_cache=True, eos_token_id=None,
                                      pad_token_id=0)
        return out[0, len(ids):].tolist()
