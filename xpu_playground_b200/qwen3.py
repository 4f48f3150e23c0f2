"""Python face of the Qwen3 decode engine (xpu_qwen3_* in include/xpu_cuda.h).

Mirrors the reference's Engine (qwen3/main.cpp:118-329): construct it for a
shape and a maximum sequence length, load weights (a seeded synthetic
checkpoint, per-tensor host uploads, or a safetensors directory through the
C++ loader), then ``decode(token, position) -> next token``. ``generate``
runs prompt + greedy generation device-resident (one host sync).
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .qwen3_config import WEIGHT_STD, Qwen3Shape

XPU_ERR_NONFINITE = _lib.XPU_ERR_NONFINITE


def shape_struct(shape: Qwen3Shape) -> _lib.Qwen3ShapeC:
    return _lib.Qwen3ShapeC(shape.hidden, shape.intermediate, shape.layers, shape.q_heads,
                            shape.kv_heads, shape.vocab, int(shape.tied), shape.eps,
                            shape.rope_theta)


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All-gather one bytes object per rank over torch.distributed, in rank order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out: list = [None] * world
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


def _shape_from_c(c: _lib.Qwen3ShapeC) -> Qwen3Shape:
    return Qwen3Shape(hidden=c.hidden_size, intermediate=c.intermediate_size, layers=c.num_hidden_layers,
                      q_heads=c.num_attention_heads, kv_heads=c.num_key_value_heads, vocab=c.vocab_size,
                      tied=bool(c.tie_word_embeddings),
                      # the C field is float32: print it back at float32 precision (1e-06, not 9.99e-07)
                      eps=float(f"{c.rms_norm_eps:.7g}"), rope_theta=c.rope_theta)


def read_config(model_dir: str) -> Qwen3Shape:
    """<model_dir>/config.json as a validated shape (xpu_qwen3_read_config)."""
    c = _lib.Qwen3ShapeC()
    _lib.check(_lib.load().xpu_qwen3_read_config(str(model_dir).encode(), ctypes.byref(c)))
    return _shape_from_c(c)


def validate_checkpoint(model_dir: str) -> tuple[Qwen3Shape, int]:
    """Config and every tensor header of a safetensors checkpoint directory,
    validated without a GPU; returns the shape and the payload bytes."""
    c = _lib.Qwen3ShapeC()
    n = ctypes.c_uint64()
    _lib.check(_lib.load().xpu_qwen3_validate_checkpoint(str(model_dir).encode(), ctypes.byref(c), ctypes.byref(n)))
    return _shape_from_c(c), n.value


class Qwen3Engine:
    def __init__(self, shape: Qwen3Shape, max_seq: int, device: int = 0, tp_rank: int = 0,
                 tp_size: int = 1, mode: str | None = None, max_batch: int = 1):
        self.lib = _lib.load()
        self.shape, self.max_seq, self.max_batch = shape, max_seq, max_batch
        self._h = ctypes.c_void_p()
        self._shape_c = shape_struct(shape)
        if max_batch != 1 and tp_size != 1:
            _lib.check(self.lib.xpu_qwen3_create_batched_tp(ctypes.byref(self._shape_c), max_seq, device, tp_rank,
                                                            tp_size, max_batch, ctypes.byref(self._h)))
        elif max_batch != 1:
            _lib.check(self.lib.xpu_qwen3_create_batched(ctypes.byref(self._shape_c), max_seq, device,
                                                         max_batch, ctypes.byref(self._h)))
        else:
            _lib.check(self.lib.xpu_qwen3_create(ctypes.byref(self._shape_c), max_seq, device, tp_rank,
                                                 tp_size, ctypes.byref(self._h)))
        if mode is not None:
            self.set_mode(mode)

    def close(self) -> None:
        if self._h:
            _lib.check(self.lib.xpu_qwen3_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------ weights ----
    def init_synthetic(self, seed: int, std: float = WEIGHT_STD) -> None:
        _lib.check(self.lib.xpu_qwen3_init_synthetic(self._h, seed, std))

    def set_tensor(self, name: str, bits: np.ndarray) -> None:
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        _lib.check(self.lib.xpu_qwen3_set_tensor(self._h, name.encode(), a.ctypes.data, a.size))

    def load_checkpoint(self, model_dir: str) -> None:
        """Streams (this rank's part of) a safetensors checkpoint directory."""
        _lib.check(self.lib.xpu_qwen3_load_checkpoint(self._h, str(model_dir).encode()))

    def load_weights(self, weights: dict[str, np.ndarray]) -> None:
        for name, bits in weights.items():
            self.set_tensor(name, bits)

    # ---------------------------------------------------- tensor parallel ----
    TP_HANDLE_BYTES = 64

    def tp_handle(self) -> bytes:
        """This rank's exchange-region handle (CUDA IPC), to be all-gathered."""
        buf = ctypes.create_string_buffer(self.TP_HANDLE_BYTES)
        _lib.check(self.lib.xpu_qwen3_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles: list[bytes]) -> None:
        """Maps the peers' exchange regions: handles[q] from rank q."""
        if any(len(h) != self.TP_HANDLE_BYTES for h in handles):
            raise ValueError("tp_connect: every handle is 64 bytes")
        blob = b"".join(handles)
        _lib.check(self.lib.xpu_qwen3_tp_connect(self._h, blob, len(handles)))

    def connect_tensor_parallel(self, group=None) -> None:
        """All-gathers the ranks' handles over a torch.distributed process
        group (any backend) and connects."""
        self.tp_connect(exchange_handles(self.tp_handle(), group))

    # ------------------------------------------------------------- decode ----
    def decode(self, token: int, position: int) -> int:
        out = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_decode(self._h, token, position, ctypes.byref(out)))
        return out.value

    def generate(self, prompt: list[int], max_new_tokens: int, stop_at_eos: bool = False) -> list[int]:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(max_new_tokens, 1), np.uint32)
        count = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_generate(self._h, p.ctypes.data, p.size, max_new_tokens,
                                               int(stop_at_eos), out.ctypes.data, ctypes.byref(count)))
        return [int(t) for t in out[:count.value]]

    def set_state(self, token: int, position: int, prompt_len: int = 0) -> None:
        _lib.check(self.lib.xpu_qwen3_set_state(self._h, token, position, prompt_len))

    def enqueue_steps(self, steps: int, stream: int | None = None) -> None:
        _lib.check(self.lib.xpu_qwen3_enqueue_steps(self._h, steps, stream))

    def state(self) -> tuple[int, int, int]:
        tok, pos, err = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_get_state(self._h, ctypes.byref(tok), ctypes.byref(pos),
                                                ctypes.byref(err)))
        return tok.value, pos.value, err.value

    def token_log(self, first_position: int, count: int) -> list[int]:
        """Greedy tokens the steps at positions [first, first + count)
        produced (xpu_qwen3_token_log)."""
        out = np.zeros(max(count, 1), np.uint32)
        _lib.check(self.lib.xpu_qwen3_token_log(self._h, first_position, count, out.ctypes.data))
        return [int(t) for t in out[:count]]

    def set_mode(self, mode: str) -> None:
        """"persistent" (one cooperative kernel per token) or "graph"."""
        _lib.check(self.lib.xpu_qwen3_set_mode(self._h, {"persistent": 0, "graph": 1}[mode]))

    def synchronize(self) -> None:
        _lib.check(self.lib.xpu_qwen3_synchronize(self._h))

    def logits(self) -> np.ndarray:
        info = self.info()
        out = np.empty(info.vocab_rows, np.uint16)
        _lib.check(self.lib.xpu_qwen3_logits(self._h, out.ctypes.data, out.size))
        return out

    def info(self) -> _lib.Qwen3InfoC:
        info = _lib.Qwen3InfoC()
        _lib.check(self.lib.xpu_qwen3_info(self._h, ctypes.byref(info)))
        return info

    def bytes_per_token(self, context: int) -> int:
        return int(self.lib.xpu_qwen3_bytes_per_token(self._h, context))

    def prefill(self, prompt: list[int]) -> int:
        """Chunked prefill (16 positions per batched step) of the batch-1
        sequence; returns the greedy token after the prompt and leaves the
        state at position len(prompt) (xpu_qwen3_prefill)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_prefill(self._h, p.ctypes.data, p.size, ctypes.byref(out)))
        return out.value

    def prefill_dense(self, prompt: list[int]) -> int:
        """Dense prefill (every position through each layer together, tcgen05
        GEMMs; xpu_qwen3_prefill_dense): returns the greedy token after the
        prompt, leaves the state at position len(prompt) and the last
        position's logits in logits()."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_prefill_dense(self._h, p.ctypes.data, p.size, ctypes.byref(out)))
        return out.value

    # ----------------------------------------------------- batched decode ----
    def batch_decode(self, tokens: list[int], positions: list[int]) -> list[int]:
        """One step of len(tokens) sequences (xpu_qwen3_batch_decode)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        if t.size != p.size:
            raise ValueError("one position per token")
        out = np.zeros(t.size, np.uint32)
        _lib.check(self.lib.xpu_qwen3_batch_decode(self._h, t.size, t.ctypes.data, p.ctypes.data,
                                                   out.ctypes.data))
        return [int(x) for x in out]

    def batch_generate(self, prompts: list[list[int]], max_new_tokens: int,
                       stop_at_eos: bool = False) -> list[list[int]]:
        """Device-resident prompts + greedy generation for len(prompts) sequences."""
        lens = np.ascontiguousarray([len(p) for p in prompts], dtype=np.uint32)
        flat = np.ascontiguousarray([t for p in prompts for t in p] or [0], dtype=np.uint32)
        out = np.zeros(max(1, len(prompts) * max_new_tokens), np.uint32)
        counts = np.zeros(len(prompts), np.uint32)
        _lib.check(self.lib.xpu_qwen3_batch_generate(self._h, len(prompts), flat.ctypes.data, lens.ctypes.data,
                                                     max_new_tokens, int(stop_at_eos), out.ctypes.data,
                                                     counts.ctypes.data))
        return [[int(x) for x in out[s * max_new_tokens: s * max_new_tokens + counts[s]]]
                for s in range(len(prompts))]

    def batch_set_state(self, tokens: list[int], positions: list[int]) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        if t.size != p.size:
            raise ValueError("one position per token")
        _lib.check(self.lib.xpu_qwen3_batch_set_state(self._h, t.size, t.ctypes.data, p.ctypes.data))

    def batch_enqueue_steps(self, steps: int, stream: int | None = None) -> None:
        _lib.check(self.lib.xpu_qwen3_batch_enqueue_steps(self._h, steps, stream))

    def batch_state(self, batch: int) -> tuple[list[int], list[int], int]:
        tok = np.zeros(batch, np.uint32)
        pos = np.zeros(batch, np.uint32)
        err = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_batch_get_state(self._h, batch, tok.ctypes.data, pos.ctypes.data,
                                                      ctypes.byref(err)))
        return [int(x) for x in tok], [int(x) for x in pos], err.value

    def batch_logits(self, sequence: int) -> np.ndarray:
        """Sequence `sequence`'s logits of the last batched step (this rank's
        vocabulary shard under tensor parallelism)."""
        out = np.empty(self.info().vocab_rows, np.uint16)
        _lib.check(self.lib.xpu_qwen3_batch_logits(self._h, sequence, out.ctypes.data, out.size))
        return out

    def batch_bytes_per_step(self, batch: int, context: int) -> int:
        return int(self.lib.xpu_qwen3_batch_bytes_per_step(self._h, batch, context))

    def batch_kernels_per_step(self) -> int:
        return int(self.lib.xpu_qwen3_batch_kernels_per_step(self._h))

    def batch_trace(self) -> np.ndarray:
        """[kernels, 8] globaltimer ns of the batched steps since the last
        call (XPU_BATCH_TRACE=1; empty otherwise), see
        xpu_qwen3_batch_trace. Resets the trace."""
        buf = np.zeros(8 * 512, np.uint64)
        n = ctypes.c_uint32()
        _lib.check(self.lib.xpu_qwen3_batch_trace(self._h, buf.ctypes.data, buf.size, ctypes.byref(n)))
        return buf[:n.value].reshape(-1, 8)
