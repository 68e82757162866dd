"""ctypes binding of libadai_b200.so (the C ABI declared in include/adai_b200.h).

Error mapping follows the reference's exceptions on the same conditions:
ADAI_B200_ERR_INVALID_ARGUMENT -> ValueError (std::invalid_argument),
ADAI_B200_ERR_OUT_OF_RANGE -> IndexError (std::out_of_range), ADAI_B200_ERR_IO -> OSError,
everything else -> RuntimeError (std::runtime_error), with DeviceTimeout / NonFiniteLogits /
NoDevice as subclasses.

There is no CPU fallback: if the library is missing, `load()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .config import ModelConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libadai_b200.so")

OK, INVALID, OUT_OF_RANGE, CUDA, TIMEOUT, NONFINITE, STATE, NO_DEVICE, IO = range(9)


class AdaiError(RuntimeError):
    pass


class DeviceTimeout(AdaiError):
    pass


class NonFiniteLogits(AdaiError):
    pass


class NoDevice(AdaiError):
    pass


class StateError(AdaiError):
    pass


EXPORTS = [
    "adai_b200_last_error", "adai_b200_ctx_create", "adai_b200_ctx_destroy",
    "adai_b200_ctx_synchronize", "adai_b200_ctx_memory", "adai_b200_ctx_stream",
    "adai_b200_model_tensor_count", "adai_b200_model_upload", "adai_b200_kv_create",
    "adai_b200_kv_destroy", "adai_b200_kv_reset", "adai_b200_kv_length", "adai_b200_encode",
    "adai_b200_decode_step", "adai_b200_generate", "adai_b200_sgemm", "adai_b200_weight_create",
    "adai_b200_weight_destroy", "adai_b200_sgemm_prepared", "adai_b200_decode_attention",
    "adai_b200_layernorm", "adai_b200_ctx_last_timing", "adai_b200_profile_step",
    "adai_b200_kv_clear_self", "adai_b200_decode_attention_static", "adai_b200_checkpoint_config",
    "adai_b200_checkpoint_read", "adai_b200_model_load", "adai_b200_gemm_strided",
    "adai_b200_softmax_rows", "adai_b200_layernorm_fwd", "adai_b200_add_row_bias",
    "adai_b200_activation", "adai_b200_embedding_gather_add_pe", "adai_b200_backend_bind",
    "adai_b200_kv_set_sampling", "adai_b200_kv_sampling_state", "adai_b200_sample_logits",
    "adai_b200_checkpoint_special_tokens", "adai_b200_ctx_check_wait_timeout",
    "adai_b200_ctx_last_work", "adai_b200_debug_sync_parse", "adai_b200_debug_configure",
    "adai_b200_debug_settings",
]

# Debug-sync modes (adai_b200_debug_configure).
SYNC_OFF, SYNC_STEP, SYNC_KERNEL = 0, 1, 2

# Kernel classes of adai_b200_profile_step (adai_b200_kernel_class).
KERNEL_CLASSES = ("gemm", "self_attention", "cross_attention", "norm", "lm_head", "other")


class Sampling(C.Structure):
    """adai_b200_sampling: GenerationConfig's sampling fields (src/TextGenerator.hpp:65-82) and the
    generator seed (0: std::random_device)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repetition_penalty", C.c_float), ("min_length", C.c_int),
                ("eos_token_id", C.c_int), ("pad_token_id", C.c_int), ("seed", C.c_uint)]

    @classmethod
    def make(cls, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, min_length=0,
             eos_token_id=3, pad_token_id=0, seed=0) -> "Sampling":
        return cls(temperature, top_k, top_p, repetition_penalty, min_length, eos_token_id,
                   pad_token_id, seed)


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("vocab", "d_model", "n_heads", "d_ff", "enc_layers", "dec_layers", "max_seq")]

    @classmethod
    def of(cls, cfg: ModelConfig) -> "ModelDesc":
        return cls(*cfg.as_cfg())


_lib = None
_vp = C.c_void_p
_ip = C.POINTER(C.c_int)


def load() -> C.CDLL:
    """Loads libadai_b200.so (built by `make -C adai_b200/csrc`); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is not built; run `make -C adai_b200/csrc` (or __graft_entry__.build())")
    lib = C.CDLL(LIB_PATH)
    lib.adai_b200_last_error.restype = C.c_char_p
    lib.adai_b200_ctx_create.argtypes = [C.c_int, C.c_float, C.POINTER(_vp)]
    lib.adai_b200_ctx_destroy.argtypes = [_vp]
    lib.adai_b200_ctx_synchronize.argtypes = [_vp, C.c_double]
    lib.adai_b200_ctx_memory.argtypes = [_vp, C.POINTER(C.c_ulonglong)]
    lib.adai_b200_ctx_check_wait_timeout.argtypes = [_vp, C.POINTER(C.c_double)]
    lib.adai_b200_ctx_last_work.argtypes = [_vp, C.c_char_p, C.c_int, C.POINTER(C.c_ulonglong)]
    lib.adai_b200_debug_sync_parse.argtypes = [C.c_char_p, _ip, C.POINTER(C.c_uint)]
    lib.adai_b200_debug_configure.argtypes = [C.c_int, C.c_uint, C.c_char_p]
    lib.adai_b200_debug_settings.argtypes = [_ip, C.POINTER(C.c_uint)]
    lib.adai_b200_ctx_stream.argtypes = [_vp]
    lib.adai_b200_ctx_stream.restype = _vp
    lib.adai_b200_model_tensor_count.argtypes = [C.POINTER(ModelDesc)]
    lib.adai_b200_model_upload.argtypes = [_vp, C.POINTER(ModelDesc), C.POINTER(_vp), _vp]
    lib.adai_b200_checkpoint_config.argtypes = [C.c_char_p, C.POINTER(ModelDesc)]
    lib.adai_b200_checkpoint_read.argtypes = [C.c_char_p, C.POINTER(ModelDesc), C.POINTER(_vp)]
    lib.adai_b200_checkpoint_special_tokens.argtypes = [C.c_char_p, _ip, _ip, _ip]
    lib.adai_b200_model_load.argtypes = [_vp, C.c_char_p, C.POINTER(ModelDesc)]
    lib.adai_b200_kv_create.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]
    lib.adai_b200_kv_destroy.argtypes = [_vp, _vp]
    lib.adai_b200_kv_reset.argtypes = [_vp, _vp, C.c_int]
    lib.adai_b200_kv_clear_self.argtypes = [_vp, _vp, C.c_int]
    lib.adai_b200_kv_length.argtypes = [_vp, _vp, C.c_int, _ip, _ip]
    lib.adai_b200_encode.argtypes = [_vp, _vp, C.c_int, _vp, _vp, _vp, _vp]
    lib.adai_b200_decode_step.argtypes = [_vp, _vp, C.c_int, _vp, _vp, _vp, _vp]
    lib.adai_b200_generate.argtypes = [_vp, _vp, C.c_int, _vp, _vp, C.c_int, _vp]
    lib.adai_b200_kv_set_sampling.argtypes = [_vp, _vp, C.c_int, C.POINTER(Sampling), _vp, C.c_int]
    lib.adai_b200_kv_sampling_state.argtypes = [_vp, _vp, C.c_int, _vp, _vp]
    lib.adai_b200_sample_logits.argtypes = [_vp, _vp, C.c_int, _vp, _vp, _vp, C.c_int, _vp]
    lib.adai_b200_sgemm.argtypes = [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp]
    lib.adai_b200_weight_create.argtypes = [_vp, _vp, C.c_int, C.c_int, C.POINTER(_vp)]
    lib.adai_b200_weight_destroy.argtypes = [_vp, _vp]
    lib.adai_b200_sgemm_prepared.argtypes = [_vp, C.c_int, _vp, _vp, _vp]
    lib.adai_b200_decode_attention.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp,
                                               _vp, _vp, _vp, C.c_int, _vp]
    lib.adai_b200_decode_attention_static.argtypes = lib.adai_b200_decode_attention.argtypes
    lib.adai_b200_layernorm.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int]
    lib.adai_b200_gemm_strided.argtypes = [_vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                           _vp, C.c_int, _vp, C.c_int, _vp, C.c_int]
    lib.adai_b200_softmax_rows.argtypes = [_vp, _vp, C.c_int, C.c_int]
    lib.adai_b200_layernorm_fwd.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                            C.c_float]
    lib.adai_b200_add_row_bias.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int]
    lib.adai_b200_activation.argtypes = [_vp, _vp, C.c_int, C.c_int]
    lib.adai_b200_embedding_gather_add_pe.argtypes = [_vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp,
                                                      C.c_int, C.c_int, C.c_int]
    lib.adai_b200_backend_bind.argtypes = [_vp]
    lib.adai_b200_ctx_last_timing.argtypes = [_vp, C.POINTER(C.c_double), _ip]
    lib.adai_b200_profile_step.argtypes = [_vp, _vp, C.c_int, _vp, _vp, C.c_int, _vp, _vp, _vp,
                                           _vp]
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc == OK:
        return
    msg = load().adai_b200_last_error().decode(errors="replace")
    if rc == INVALID:
        raise ValueError(msg)
    if rc == OUT_OF_RANGE:
        raise IndexError(msg)
    if rc == TIMEOUT:
        raise DeviceTimeout(msg)
    if rc == NONFINITE:
        raise NonFiniteLogits(msg)
    if rc == NO_DEVICE:
        raise NoDevice(msg)
    if rc == STATE:
        raise StateError(msg)
    if rc == IO:
        raise OSError(msg)
    raise AdaiError(msg)


def debug_sync_parse(value: str | None) -> tuple[int, int]:
    """(mode, every) of an ADAI_B200_SYNC value; ValueError for one the library cannot read."""
    m, e = C.c_int(), C.c_uint()
    check(load().adai_b200_debug_sync_parse(None if value is None else value.encode(), C.byref(m),
                                            C.byref(e)))
    return m.value, e.value


def debug_configure(mode: int = SYNC_OFF, every: int = 1, trace_file: str | None = None) -> None:
    """Replaces the process's debug-sync settings (ADAI_B200_SYNC / ADAI_B200_TRACE_FILE)."""
    check(load().adai_b200_debug_configure(mode, every,
                                           None if trace_file is None else os.fsencode(trace_file)))


def debug_settings() -> tuple[int, int]:
    m, e = C.c_int(), C.c_uint()
    check(load().adai_b200_debug_settings(C.byref(m), C.byref(e)))
    return m.value, e.value


def checkpoint_config(directory: str) -> ModelConfig:
    """The model shape of a checkpoint: a SafeTensors directory or a save_model prefix (host
    only)."""
    d = ModelDesc()
    check(load().adai_b200_checkpoint_config(os.fsencode(directory), C.byref(d)))
    return ModelConfig(d.vocab, d.d_model, d.n_heads, d.d_ff, d.enc_layers, d.dec_layers,
                       d.max_seq)


def checkpoint_special_tokens(path: str) -> tuple[int, int, int]:
    """(BOS, EOS, PAD) of a checkpoint (host only)."""
    b, e, p = C.c_int(), C.c_int(), C.c_int()
    check(load().adai_b200_checkpoint_special_tokens(os.fsencode(path), C.byref(b), C.byref(e),
                                                     C.byref(p)))
    return b.value, e.value, p.value


def read_checkpoint(directory: str, cfg: ModelConfig | None = None) -> list[np.ndarray]:
    """The tensors of a SafeTensors checkpoint in the model-upload order and layouts, read by
    the library's own reader (host only)."""
    from .synth import tensor_specs
    cfg = cfg or checkpoint_config(directory)
    out = [np.empty(shape, np.float32) for _, shape in tensor_specs(cfg)]
    arr = (_vp * len(out))(*[o.ctypes.data for o in out])
    check(load().adai_b200_checkpoint_read(os.fsencode(directory), C.byref(ModelDesc.of(cfg)), arr))
    return out


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a):
    return None if a is None else a.ctypes.data


class Context:
    """One GPU (the reference GPUManager's device + stream). Use one per device, one host thread
    at a time."""

    def __init__(self, device: int = 0, mem_fraction: float = 0.0):
        self.lib = load()
        h = _vp()
        check(self.lib.adai_b200_ctx_create(device, mem_fraction, C.byref(h)))
        self.h = h
        self.device = device
        self.cfg: ModelConfig | None = None

    def close(self) -> None:
        if getattr(self, "h", None):
            check(self.lib.adai_b200_ctx_destroy(self.h))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return self.lib.adai_b200_ctx_stream(self.h) or 0

    def synchronize(self, timeout_s: float = 0.0) -> None:
        check(self.lib.adai_b200_ctx_synchronize(self.h, timeout_s))

    def check_wait_timeout(self) -> float:
        """Makes one bounded device wait run out on purpose and returns the wall seconds the call
        took. The expected outcome is the library's timeout status, after which this context is
        unusable; any other status raises."""
        t = C.c_double()
        rc = self.lib.adai_b200_ctx_check_wait_timeout(self.h, C.byref(t))
        if rc != TIMEOUT:
            check(rc)
            raise AdaiError("the device wait did not report a timeout")
        return t.value

    def last_work(self) -> tuple[str, int]:
        """("<seq> <phase> <kernel>", seq) of the last GPU work this context queued."""
        buf = C.create_string_buffer(256)
        n = C.c_ulonglong()
        check(self.lib.adai_b200_ctx_last_work(self.h, buf, len(buf), C.byref(n)))
        return buf.value.decode(), n.value

    def memory_bytes(self) -> int:
        v = C.c_ulonglong()
        check(self.lib.adai_b200_ctx_memory(self.h, C.byref(v)))
        return v.value

    def upload(self, cfg: ModelConfig, weights, pe_table=None) -> None:
        ws = [np.ascontiguousarray(w, np.float32) for w in weights]
        desc = ModelDesc.of(cfg)
        n = self.lib.adai_b200_model_tensor_count(C.byref(desc))
        if n != len(ws):
            raise ValueError(f"model needs {n} tensors, got {len(ws)}")
        arr = (_vp * len(ws))(*[w.ctypes.data for w in ws])
        pe = None if pe_table is None else np.ascontiguousarray(pe_table, np.float32)
        check(self.lib.adai_b200_model_upload(self.h, C.byref(desc), arr, _ptr(pe)))
        self.cfg = cfg

    def load(self, directory: str, expect: ModelConfig | None = None) -> ModelConfig:
        """Loads a SafeTensors checkpoint directory (config.json + model.safetensors, the
        reference's ModelSerializer layout); with `expect`, its shape must match."""
        exp = C.byref(ModelDesc.of(expect)) if expect is not None else None
        check(self.lib.adai_b200_model_load(self.h, os.fsencode(directory), exp))
        self.cfg = checkpoint_config(directory)
        return self.cfg

    def kv_arena(self, max_slots: int, self_capacity: int, cross_capacity: int) -> "KVArena":
        return KVArena(self, max_slots, self_capacity, cross_capacity)

    # ---- op level (device pointers: ints, e.g. torch tensor .data_ptr()) ----
    def sgemm(self, m, n, k, A_ptr, B_ptr, C_ptr) -> None:
        check(self.lib.adai_b200_sgemm(self.h, m, n, k, A_ptr, B_ptr, C_ptr))

    def weight(self, B_ptr, k, n) -> "PreparedWeight":
        return PreparedWeight(self, B_ptr, k, n)

    def decode_attention(self, B, H, capacity, q, k_new, v_new, k_cache, v_cache, lens, max_len,
                         out, head_dim=64) -> None:
        check(self.lib.adai_b200_decode_attention(self.h, B, H, head_dim, capacity, q, k_new,
                                                  v_new, k_cache, v_cache, lens, max_len, out))

    def decode_attention_static(self, B, H, capacity, q, k_new, v_new, k_cache, v_cache, lens,
                                max_len, out, head_dim=64) -> None:
        """decode_attention without any device allocation: the split-KV scratch is a fixed
        16 MiB array per device, shared by every caller on that device (calls that overlap in
        time race). Too-large calls raise IndexError."""
        check(self.lib.adai_b200_decode_attention_static(self.h, B, H, head_dim, capacity, q,
                                                         k_new, v_new, k_cache, v_cache, lens,
                                                         max_len, out))

    def layernorm(self, x, gamma, beta, out, rows, D) -> None:
        check(self.lib.adai_b200_layernorm(self.h, x, gamma, beta, out, rows, D))

    # ---- the reference backend table's decode-path entries (device pointers) ----
    def gemm_strided(self, trans_a, trans_b, m, n, k, alpha, a, lda, b, ldb, c, ldc) -> None:
        check(self.lib.adai_b200_gemm_strided(self.h, int(trans_a), int(trans_b), m, n, k, alpha,
                                              a, lda, b, ldb, c, ldc))

    def softmax_rows(self, data, rows, cols) -> None:
        check(self.lib.adai_b200_softmax_rows(self.h, data, rows, cols))

    def layernorm_fwd(self, x, y, x_normed, gamma, beta, mean, rstd, rows, cols, eps=1e-5) -> None:
        check(self.lib.adai_b200_layernorm_fwd(self.h, x, y, x_normed, gamma, beta, mean, rstd,
                                               rows, cols, eps))

    def add_row_bias(self, m, bias, out, rows, cols) -> None:
        check(self.lib.adai_b200_add_row_bias(self.h, m, bias, out, rows, cols))

    def activation(self, data, size, kind) -> None:
        """kind: 0 ReLU, 1 sigmoid, 2 tanh, 3 GELU (tanh form)."""
        check(self.lib.adai_b200_activation(self.h, data, size, kind))

    def embedding_gather_add_pe(self, table, ids, pe, pe_rows, pos_offset, out, n, d, vocab=0):
        check(self.lib.adai_b200_embedding_gather_add_pe(self.h, table, ids, pe, pe_rows,
                                                         pos_offset, out, n, d, vocab))

    def bind_backend(self) -> None:
        """Makes this context the one the adai::gpu::matrix_*_gpu C++ functions run on."""
        check(self.lib.adai_b200_backend_bind(self.h))

    def last_timing(self) -> tuple[float, int]:
        """(device ms of the last generate() decode loop, kernels launched per step)."""
        ms, k = C.c_double(), C.c_int()
        check(self.lib.adai_b200_ctx_last_timing(self.h, C.byref(ms), C.byref(k)))
        return ms.value, k.value


class PreparedWeight:
    def __init__(self, ctx: Context, B_ptr, k, n):
        self.ctx, self.k, self.n = ctx, k, n
        h = _vp()
        check(ctx.lib.adai_b200_weight_create(ctx.h, B_ptr, k, n, C.byref(h)))
        self.h = h

    def matmul(self, m, A_ptr, C_ptr) -> None:
        check(self.ctx.lib.adai_b200_sgemm_prepared(self.ctx.h, m, A_ptr, self.h, C_ptr))

    def close(self):
        if getattr(self, "h", None):
            check(self.ctx.lib.adai_b200_weight_destroy(self.ctx.h, self.h))
            self.h = None


class KVArena:
    """Per-sequence self/cross caches for `max_slots` sequences (the reference DecoderKVCache,
    one per slot), plus the decode entry points that use them."""

    def __init__(self, ctx: Context, max_slots: int, self_capacity: int, cross_capacity: int):
        self.ctx, self.lib = ctx, ctx.lib
        self.max_slots = max_slots
        self.self_capacity = self_capacity
        self.cross_capacity = cross_capacity
        h = _vp()
        check(self.lib.adai_b200_kv_create(ctx.h, max_slots, self_capacity, cross_capacity,
                                           C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            check(self.lib.adai_b200_kv_destroy(self.ctx.h, self.h))
        self.h = None

    def reset(self, slot: int) -> None:
        check(self.lib.adai_b200_kv_reset(self.ctx.h, self.h, slot))

    def clear_self(self, slot: int) -> None:
        check(self.lib.adai_b200_kv_clear_self(self.ctx.h, self.h, slot))

    def length(self, slot: int) -> tuple[int, int]:
        a, b = C.c_int(), C.c_int()
        check(self.lib.adai_b200_kv_length(self.ctx.h, self.h, slot, C.byref(a), C.byref(b)))
        return a.value, b.value

    def encode(self, slots, sources, want_output=False):
        """Encoder prefill of each source (a list of id arrays) into its slot."""
        slots = _i32(slots)
        lens = _i32([len(s) for s in sources])
        ids = _i32(np.concatenate([np.asarray(s, np.int32) for s in sources]))
        out = (np.empty((int(lens.sum()), self.ctx.cfg.d_model), np.float32)
               if want_output else None)
        check(self.lib.adai_b200_encode(self.ctx.h, self.h, len(slots), _ptr(slots), _ptr(ids),
                                        _ptr(lens), _ptr(out)))
        return out

    def decode_step(self, slots, ids, want_logits=False):
        slots, ids = _i32(slots), _i32(ids)
        B = slots.size
        nxt = np.empty(B, np.int32)
        lg = np.empty((B, self.ctx.cfg.vocab), np.float32) if want_logits else None
        check(self.lib.adai_b200_decode_step(self.ctx.h, self.h, B, _ptr(slots), _ptr(ids),
                                             _ptr(nxt), _ptr(lg)))
        return nxt, lg

    def profile_step(self, slots, ids) -> dict:
        """One eager decode step with CUDA events around every kernel; per kernel class:
        ms, algorithmic bytes, flops, launches."""
        slots, ids = _i32(slots), _i32(ids)
        n = len(KERNEL_CLASSES)
        ms, by, fl = (np.zeros(n, np.float64) for _ in range(3))
        ln = np.zeros(n, np.int32)
        check(self.lib.adai_b200_profile_step(self.ctx.h, self.h, slots.size, _ptr(slots),
                                              _ptr(ids), n, _ptr(ms), _ptr(by), _ptr(fl),
                                              _ptr(ln)))
        return {k: dict(ms=float(ms[i]), bytes=float(by[i]), flops=float(fl[i]),
                        launches=int(ln[i])) for i, k in enumerate(KERNEL_CLASSES)}

    def set_sampling(self, slot: int, cfg: "Sampling | None", history=()) -> None:
        """Configures slot for the reference's sampling rules (None: back to the argmax)."""
        h = _i32(list(history))
        check(self.lib.adai_b200_kv_set_sampling(self.ctx.h, self.h, slot,
                                                 C.byref(cfg) if cfg is not None else None,
                                                 _ptr(h) if h.size else None, h.size))

    def sampling_state(self, slot: int) -> tuple[np.ndarray, int]:
        """(std::mt19937 state words [625]: 624 state + read position, steps sampled)."""
        st = np.zeros(625, np.uint32)
        n = C.c_int()
        check(self.lib.adai_b200_kv_sampling_state(self.ctx.h, self.h, slot, _ptr(st),
                                                   C.byref(n)))
        return st, n.value

    def sample_logits(self, slots, logits_ptr, ld, fed_ids=None) -> np.ndarray:
        """Tokens for device logits rows [B, ld] by each slot's sampling rules."""
        slots = _i32(slots)
        fed = _i32(fed_ids) if fed_ids is not None else None
        nxt = np.empty(slots.size, np.int32)
        check(self.lib.adai_b200_sample_logits(self.ctx.h, self.h, slots.size, _ptr(slots),
                                               _ptr(fed), logits_ptr, ld, _ptr(nxt)))
        return nxt

    def generate(self, slots, first_ids, steps):
        slots, first = _i32(slots), _i32(first_ids)
        out = np.empty((slots.size, steps), np.int32)
        check(self.lib.adai_b200_generate(self.ctx.h, self.h, slots.size, _ptr(slots),
                                          _ptr(first), steps, _ptr(out)))
        return out
