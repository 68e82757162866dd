"""ctypes wrappers over the two CPU oracles. TEST INFRASTRUCTURE ONLY.

* `Port`  — oracle/liboracle_port.so, the plain-C restatement (oracle/adai_oracle.c).
* `Ref`   — oracle/_ref/libadai_ref.so, the reference's own sources built by oracle/Makefile
            with our driver (oracle/ref_driver.cpp). Present wherever it was built (it travels
            with the repository snapshot as a built file); `Ref.available()` says whether it is.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "liboracle_port.so")
REF_SO = os.path.join(HERE, "_ref", "libadai_ref.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build_port() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)


def _ptr_array(ws):
    arr = (C.c_void_p * len(ws))()
    for i, w in enumerate(ws):
        assert w.dtype == np.float32 and w.flags.c_contiguous
        arr[i] = w.ctypes.data
    return arr


def sampling_cfg(temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, min_length=0,
                 eos=3, pad=0, bos=2):
    """GenerationConfig's sampling fields (src/TextGenerator.hpp:65-82) as the oracles take them:
    fcfg = {temperature, top_p, repetition_penalty}, icfg = {top_k, min_length, eos, pad, bos}."""
    return (np.array([temperature, top_p, repetition_penalty], np.float32),
            np.array([top_k, min_length, eos, pad, bos], np.int32))


class _Base:
    lib: C.CDLL

    def matmul(self, A, B):
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        M, K = A.shape
        K2, N = B.shape
        assert K == K2
        out = np.empty((M, N), np.float32)
        self._check(getattr(self.lib, self._p + "matmul")(A, B, out, M, K, N))
        return out

    def _check(self, rc):
        if rc not in (None, 0):
            raise RuntimeError(f"oracle call failed: {self._err()}")

    def _err(self):
        return "error"


class Port(_Base):
    _p = "orc_"

    def __init__(self):
        if not os.path.exists(PORT_SO):
            build_port()
        lib = C.CDLL(PORT_SO)
        lib.orc_matmul.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.orc_matmul.restype = None
        lib.orc_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int]
        lib.orc_gelu.argtypes = [_f32p, _f32p, C.c_int]
        lib.orc_softmax_row.argtypes = [_f32p, _f32p, C.c_int]
        lib.orc_pe_table.argtypes = [C.c_int, C.c_int, _f32p]
        lib.orc_attention_single.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                             _f32p]
        lib.orc_argmax.argtypes = [_f32p, C.c_int]
        lib.orc_argmax.restype = C.c_int
        lib.orc_model_create.argtypes = [_i32p, C.c_void_p]
        lib.orc_model_create.restype = C.c_void_p
        lib.orc_model_destroy.argtypes = [C.c_void_p]
        lib.orc_encode.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p]
        lib.orc_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                     _i32p, C.c_void_p]
        _u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        _u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        _f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
        lib.orc_mt_seed.argtypes = [_u32p, C.c_uint]
        lib.orc_mt_next.argtypes = [_u32p]
        lib.orc_mt_next.restype = C.c_uint
        lib.orc_canonical.argtypes = [_u32p]
        lib.orc_canonical.restype = C.c_double
        lib.orc_sample_next.argtypes = [_f32p, C.c_int, _f32p, _i32p, _u8p, C.c_int, _u32p,
                                        C.POINTER(C.c_double)]
        lib.orc_sample_next.restype = C.c_int
        lib.orc_sample_generate.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i32p, C.c_uint,
                                            C.c_void_p, C.c_int, _i32p, _f64p]
        lib.orc_sample_generate.restype = C.c_int
        self.lib = lib

    # ---- sampling (TextGenerator::generate) ----
    def mt_seed(self, seed):
        st = np.zeros(625, np.uint32)
        self.lib.orc_mt_seed(st, seed)
        return st

    def mt_next(self, st):
        return int(self.lib.orc_mt_next(st))

    def canonical(self, st):
        return float(self.lib.orc_canonical(st))

    def sample_next(self, row, cfg, seen, new_tokens, st):
        """One token from a logits row; seen is a uint8 [V] mask; st an mt19937 state that the
        call advances. Returns (token, margin); token < 0 for the next_logits errors."""
        row = np.ascontiguousarray(row, np.float32)
        m = C.c_double(0.0)
        tok = self.lib.orc_sample_next(row, row.size, cfg[0], cfg[1],
                                       np.ascontiguousarray(seen, np.uint8), int(new_tokens), st,
                                       C.byref(m))
        return int(tok), m.value

    def sample_generate(self, logits, cfg, seed, prompt=None):
        """TextGenerator(cfg, seed).generate over the rows of logits [steps, V]: (sequence with
        its start tokens, per-step margins)."""
        logits = np.ascontiguousarray(logits, np.float32)
        steps, V = logits.shape
        pr = np.ascontiguousarray(prompt if prompt is not None else [], np.int32)
        out = np.empty(max(pr.size, 1) + steps, np.int32)
        margins = np.full(steps, np.nan)
        n = self.lib.orc_sample_generate(logits, V, steps, cfg[0], cfg[1], seed,
                                         pr.ctypes.data if pr.size else None, pr.size, out, margins)
        if n < 0:
            raise ValueError("sample_generate: non-finite logits" if n == -1 else
                             "sample_generate: every logit is -inf")
        return out[:n].copy(), margins

    def layernorm(self, x, g, b):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.orc_layernorm(x, np.ascontiguousarray(g, np.float32),
                               np.ascontiguousarray(b, np.float32), out, x.shape[0], x.shape[1])
        return out

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        self.lib.orc_gelu(x, out, x.size)
        return out

    def softmax_rows(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        for i in range(x.shape[0]):
            r = np.ascontiguousarray(x[i])
            o = np.empty_like(r)
            self.lib.orc_softmax_row(r, o, r.size)
            out[i] = o
        return out

    def pe_table(self, max_len, D):
        out = np.empty((max_len, D), np.float32)
        self.lib.orc_pe_table(max_len, D, out)
        return out

    def attention_single(self, q, K, V, H):
        q = np.ascontiguousarray(q, np.float32)
        K = np.ascontiguousarray(K, np.float32)
        V = np.ascontiguousarray(V, np.float32)
        out = np.empty_like(q)
        self.lib.orc_attention_single(q, K, V, K.shape[0], K.shape[1], H, out)
        return out

    def model(self, cfg, weights):
        return _PortModel(self, cfg, weights)


class _PortModel:
    def __init__(self, port, cfg, weights):
        self.port, self.cfg = port, cfg
        self.weights = [np.ascontiguousarray(w, np.float32) for w in weights]
        self._ptrs = _ptr_array(self.weights)
        self.h = port.lib.orc_model_create(np.asarray(cfg.as_cfg(), np.int32), self._ptrs)
        if not self.h:
            raise ValueError("bad model config")

    def __del__(self):
        if getattr(self, "h", None):
            self.port.lib.orc_model_destroy(self.h)
            self.h = None

    def encode(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, self.cfg.d_model), np.float32)
        if self.port.lib.orc_encode(self.h, ids, ids.size, out) != 0:
            raise ValueError("encode failed")
        return out

    def generate(self, src, steps, bos=2, forced=None, want_logits=False):
        src = np.ascontiguousarray(src, np.int32)
        ids = np.empty(steps, np.int32)
        lg = np.empty((steps, self.cfg.vocab), np.float32) if want_logits else None
        fz = np.ascontiguousarray(forced, np.int32) if forced is not None else None
        rc = self.port.lib.orc_generate(self.h, src, src.size, bos, steps,
                                        fz.ctypes.data if fz is not None else None, ids,
                                        lg.ctypes.data if lg is not None else None)
        if rc != 0:
            raise ValueError("generate failed")
        return ids, lg


class Ref(_Base):
    _p = "ref_"

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def __init__(self):
        if not self.available():
            raise FileNotFoundError(REF_SO)
        lib = C.CDLL(REF_SO)
        lib.ref_last_error.restype = C.c_char_p
        lib.ref_matmul_kernel.restype = C.c_char_p
        lib.ref_matmul.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]
        lib.ref_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int]
        lib.ref_gelu.argtypes = [_f32p, _f32p, C.c_int]
        lib.ref_softmax_rows.argtypes = [_f32p, _f32p, C.c_int, C.c_int]
        lib.ref_pe_table.argtypes = [C.c_int, C.c_int, _f32p]
        lib.ref_attention_single.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                             _f32p]
        lib.ref_model_create.argtypes = [_i32p, C.c_void_p, C.POINTER(C.c_void_p)]
        lib.ref_model_destroy.argtypes = [C.c_void_p]
        lib.ref_generate_timed.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p,
                                           np.ctypeslib.ndpointer(np.float64,
                                                                  flags="C_CONTIGUOUS"),
                                           C.POINTER(C.c_double)]
        lib.ref_generate_timed_threads.argtypes = [
            C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, _i32p, _i32p,
            np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS"), C.POINTER(C.c_double)]
        lib.ref_encode.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p]
        lib.ref_generate.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                     _i32p, C.c_void_p, C.POINTER(C.c_double),
                                     C.POINTER(C.c_double)]
        _f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
        lib.ref_generate_hidden.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int,
                                            C.c_void_p, _i32p, _f32p, _f64p, _f32p]
        lib.ref_sample_generate.argtypes = [_f32p, C.c_int, C.c_int, _f32p, _i32p, C.c_uint,
                                            C.c_void_p, C.c_int, _i32p, C.POINTER(C.c_int)]
        lib.ref_model_save.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_int]
        self.lib = lib

    def sample_generate(self, logits, cfg, seed, prompt=None):
        """The reference's TextGenerator(cfg, seed).generate over the rows of logits."""
        logits = np.ascontiguousarray(logits, np.float32)
        steps, V = logits.shape
        pr = np.ascontiguousarray(prompt if prompt is not None else [], np.int32)
        out = np.empty(max(pr.size, 1) + steps, np.int32)
        n = C.c_int(0)
        self._check(self.lib.ref_sample_generate(logits, V, steps, cfg[0], cfg[1], seed,
                                                 pr.ctypes.data if pr.size else None, pr.size,
                                                 out, C.byref(n)))
        return out[:n.value].copy()

    def _err(self):
        return self.lib.ref_last_error().decode()

    def matmul_kernel(self) -> str:
        return self.lib.ref_matmul_kernel().decode()

    def layernorm(self, x, g, b):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.ref_layernorm(x, np.ascontiguousarray(g, np.float32),
                                           np.ascontiguousarray(b, np.float32), out,
                                           x.shape[0], x.shape[1]))
        return out

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.empty_like(x)
        self._check(self.lib.ref_gelu(x, out, x.size))
        return out

    def softmax_rows(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.ref_softmax_rows(x, out, x.shape[0], x.shape[1]))
        return out

    def pe_table(self, max_len, D):
        out = np.empty((max_len, D), np.float32)
        self._check(self.lib.ref_pe_table(max_len, D, out))
        return out

    def attention_single(self, q, K, V, H):
        q = np.ascontiguousarray(q, np.float32)
        K = np.ascontiguousarray(K, np.float32)
        V = np.ascontiguousarray(V, np.float32)
        out = np.empty_like(q)
        self._check(self.lib.ref_attention_single(q, K, V, K.shape[0], K.shape[1], H, out))
        return out

    def model(self, cfg, weights):
        return _RefModel(self, cfg, weights)


class _RefModel:
    def __init__(self, ref, cfg, weights):
        self.ref, self.cfg = ref, cfg
        ws = [np.ascontiguousarray(w, np.float32) for w in weights]
        h = C.c_void_p()
        ref._check(ref.lib.ref_model_create(np.asarray(cfg.as_cfg(), np.int32), _ptr_array(ws),
                                            C.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_model_destroy(self.h)
            self.h = None

    def encode(self, ids):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, self.cfg.d_model), np.float32)
        self.ref._check(self.ref.lib.ref_encode(self.h, ids, ids.size, out))
        return out

    def save(self, prefix, bos=2, eos=3, pad=0):
        """The reference's own checkpoint files (EncoderDecoderModel::save_model layout)."""
        self.ref._check(self.ref.lib.ref_model_save(self.h, os.fsencode(prefix), bos, eos, pad))

    def generate_hidden(self, src, steps, bos=2, forced=None):
        """Greedy decode returning (ids, hidden [steps, D], float64 logit-row sums, top-2 logits
        [steps, 2]); hidden is the decoder output row the head multiplies."""
        src = np.ascontiguousarray(src, np.int32)
        ids = np.empty(steps, np.int32)
        hid = np.empty((steps, self.cfg.d_model), np.float32)
        sums = np.empty(steps, np.float64)
        top2 = np.empty((steps, 2), np.float32)
        fz = np.ascontiguousarray(forced, np.int32) if forced is not None else None
        self.ref._check(self.ref.lib.ref_generate_hidden(
            self.h, src, src.size, bos, steps, fz.ctypes.data if fz is not None else None, ids,
            hid, sums, top2))
        return ids, hid, sums, top2

    def generate_timed(self, src, steps, bos=2):
        """Greedy decode; returns (ids, per-step wall seconds, encoder seconds)."""
        src = np.ascontiguousarray(src, np.int32)
        ids = np.empty(steps, np.int32)
        st = np.empty(steps, np.float64)
        te = C.c_double()
        self.ref._check(self.ref.lib.ref_generate_timed(self.h, src, src.size, bos, steps, ids,
                                                        st, C.byref(te)))
        return ids, st, te.value

    def generate_timed_threads(self, src, threads, bos=2):
        """Greedy decode of len(threads) steps, step s on threads[s] OpenMP threads (0: the
        default team); returns (ids, per-step wall seconds, encoder seconds)."""
        src = np.ascontiguousarray(src, np.int32)
        th = np.ascontiguousarray(threads, np.int32)
        ids = np.empty(th.size, np.int32)
        st = np.empty(th.size, np.float64)
        te = C.c_double()
        self.ref._check(self.ref.lib.ref_generate_timed_threads(
            self.h, src, src.size, bos, th.size, th, ids, st, C.byref(te)))
        return ids, st, te.value

    def generate(self, src, steps, bos=2, forced=None, want_logits=False, timings=None):
        src = np.ascontiguousarray(src, np.int32)
        ids = np.empty(steps, np.int32)
        lg = np.empty((steps, self.cfg.vocab), np.float32) if want_logits else None
        fz = np.ascontiguousarray(forced, np.int32) if forced is not None else None
        te, td = C.c_double(), C.c_double()
        self.ref._check(self.ref.lib.ref_generate(
            self.h, src, src.size, bos, steps, fz.ctypes.data if fz is not None else None, ids,
            lg.ctypes.data if lg is not None else None, C.byref(te), C.byref(td)))
        if timings is not None:
            timings["encode_s"] = te.value
            timings["decode_s"] = td.value
        return ids, lg
