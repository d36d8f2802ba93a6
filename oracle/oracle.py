"""ctypes binding of the CPU oracle and of the reference's own CPU kernels.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product package.

Seeded synthetic inputs are generated here too (``gaussian``), so every test,
fixture and bench run builds the same weights from the same seeds.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 8, 12, 13, 14
QTYPES = {"Q4_0": Q4_0, "Q8_0": Q8_0, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}
QNAMES = {v: k for k, v in QTYPES.items()}
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}

_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64


class ModelCfg(ctypes.Structure):
    """oracle_model_cfg (hesa_oracle.h)."""
    _fields_ = [(n, _i64) for n in ("n_layer", "d_model", "n_head", "n_kv_head", "head_dim", "d_ff", "vocab",
                                    "ctx")] + [("rms_eps", ctypes.c_float), ("rope_base", ctypes.c_float),
                                               ("qtype", ctypes.c_int)]


class LayerPtrs(ctypes.Structure):
    """oracle_layer (hesa_oracle.h)."""
    _fields_ = [(n, _vp) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm", "ffn_norm",
                                   "k_cache", "v_cache")]


def _p(a: np.ndarray, t=_vp):
    return ctypes.cast(a.ctypes.data, t)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build_oracle()
        L = ctypes.CDLL(path)
        L.oracle_fp16_to_fp32.restype = ctypes.c_float
        L.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.oracle_fp32_to_fp16.restype = ctypes.c_uint16
        L.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.oracle_row_bytes.restype = ctypes.c_size_t
        L.oracle_row_bytes.argtypes = [ctypes.c_int, _i64]
        L.oracle_dequantize_row.argtypes = [ctypes.c_int, _vp, _f32p, _i64]
        L.oracle_quantize_row.argtypes = [ctypes.c_int, _f32p, _vp, _i64]
        L.oracle_qmatvec.argtypes = [ctypes.c_int, _vp, _i64, _i64, _f32p, _i64, _i64,
                                     _f32p, _i64, ctypes.c_float, ctypes.c_int]
        L.oracle_rms_norm.argtypes = [_f32p, _f32p, _f32p, _i64, ctypes.c_float]
        L.oracle_silu_mul.argtypes = [_f32p, _f32p, _f32p, _i64]
        L.oracle_rope.argtypes = [_f32p, ctypes.c_int32, _i64, _i64, ctypes.c_float]
        L.oracle_rope_table.argtypes = [_f32p, _f32p, ctypes.c_int32, _i64, ctypes.c_float]
        L.oracle_attention_f16kv.argtypes = [_f32p, _u16p, _u16p, _f32p, _i64, _i64, _i64,
                                             _i64, ctypes.c_int]
        L.oracle_decode_step.argtypes = [ctypes.POINTER(ModelCfg), ctypes.POINTER(LayerPtrs), _f32p, _vp,
                                         _f32p, ctypes.c_int32, _f32p, ctypes.c_int]
        L.oracle_decode_step_f64.argtypes = L.oracle_decode_step.argtypes
        _lib = L
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own CPU kernels (oracle/_ref), or None if unavailable."""
    global _ref
    if _ref is None:
        path = _build.build_ref()
        if path is None or not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_cpu_matmul_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_float]
        L.ref_cpu_matvec_mt.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_int]
        L.ref_cpu_rms_norm_f32.argtypes = [_f32p, _f32p, _f32p, ctypes.c_size_t,
                                           ctypes.c_size_t, ctypes.c_float]
        L.ref_cpu_silu_f32.argtypes = [_f32p, _f32p, ctypes.c_size_t]
        L.ref_cpu_softmax_f32.argtypes = [_f32p, _f32p, ctypes.c_size_t, ctypes.c_size_t]
        L.ref_cpu_rope_f32.argtypes = [_f32p, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t,
                                       ctypes.c_size_t, ctypes.c_size_t, ctypes.c_float]
        _ref = L
    return _ref


def n_threads_default() -> int:
    return max(1, len(os.sched_getaffinity(0)))


# --------------------------------------------------------------------------
# Seeded synthetic data
# --------------------------------------------------------------------------

def gaussian(shape, std: float, seed: int) -> np.ndarray:
    """fp32 N(0, std^2) from numpy's PCG64 with the given seed."""
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def row_bytes(qtype: int, k: int) -> int:
    return (k // BLOCK_ELEMS[qtype]) * BLOCK_BYTES[qtype]


# --------------------------------------------------------------------------
# Codec
# --------------------------------------------------------------------------

def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    """Quantize fp32 [rows, k] into packed uint8 [rows, row_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    out = np.empty((rows, row_bytes(qtype, k)), dtype=np.uint8)
    L = lib()
    flat = w.reshape(-1)
    if L.oracle_quantize_row(qtype, _p(flat, _f32p), _p(out), rows * k) != 0:
        raise ValueError("oracle_quantize_row failed")
    return out


def dequantize(qtype: int, blocks: np.ndarray, k: int) -> np.ndarray:
    """Decode packed uint8 [rows, row_bytes] into fp32 [rows, k]."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    rows = blocks.shape[0]
    out = np.empty((rows, k), dtype=np.float32)
    if lib().oracle_dequantize_row(qtype, _p(blocks), _p(out, _f32p), rows * k) != 0:
        raise ValueError("oracle_dequantize_row failed")
    return out


def qmatvec(qtype: int, w: np.ndarray, x: np.ndarray, scale: float = 1.0,
            n_threads: int | None = None) -> np.ndarray:
    """y[b, n] = scale * sum_k deq(W[n, k]) x[b, k]; x is [k] or [B, k]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    B, k = x2.shape
    n_out = w.shape[0]
    y = np.empty((B, n_out), dtype=np.float32)
    rc = lib().oracle_qmatvec(qtype, _p(w), n_out, k, _p(x2, _f32p), k, B, _p(y, _f32p), n_out,
                              float(scale), n_threads or n_threads_default())
    if rc != 0:
        raise ValueError("oracle_qmatvec failed")
    return y if np.ndim(x) == 2 else y[0]


def fp32_to_fp16_bits(a: np.ndarray) -> np.ndarray:
    L = lib()
    flat = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    return np.array([L.oracle_fp32_to_fp16(float(v)) for v in flat], dtype=np.uint16).reshape(np.shape(a))


# --------------------------------------------------------------------------
# Decode-step primitives
# --------------------------------------------------------------------------

def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_rms_norm(_p(x, _f32p), _p(w, _f32p), _p(out, _f32p), x.size, float(eps))
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().oracle_silu_mul(_p(g, _f32p), _p(u, _f32p), _p(out, _f32p), g.size)
    return out


def rope(x: np.ndarray, pos: int, n_heads: int, head_dim: int, base: float = 10000.0) -> np.ndarray:
    out = np.array(x, dtype=np.float32, copy=True)
    lib().oracle_rope(_p(out, _f32p), int(pos), n_heads, head_dim, float(base))
    return out


def rope_table(pos: int, head_dim: int, base: float = 10000.0):
    c = np.empty(head_dim // 2, dtype=np.float32)
    s = np.empty(head_dim // 2, dtype=np.float32)
    lib().oracle_rope_table(_p(c, _f32p), _p(s, _f32p), int(pos), head_dim, float(base))
    return c, s


def attention_f16kv(q, k_cache, v_cache, n_head, n_kv_head, head_dim, n_ctx,
                    n_threads: int | None = None) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_cache = np.ascontiguousarray(k_cache, dtype=np.uint16)
    v_cache = np.ascontiguousarray(v_cache, dtype=np.uint16)
    out = np.empty(n_head * head_dim, dtype=np.float32)
    lib().oracle_attention_f16kv(_p(q, _f32p), _p(k_cache, _u16p), _p(v_cache, _u16p),
                                 _p(out, _f32p), n_head, n_kv_head, head_dim, n_ctx,
                                 n_threads or n_threads_default())
    return out


def decode_step(cfg: dict, layers: list, out_norm: np.ndarray, w_out: np.ndarray, x_in: np.ndarray, pos: int,
                n_threads: int | None = None, f64: bool = False) -> np.ndarray:
    """oracle_decode_step: logits of one token. `layers` holds dicts of numpy
    arrays (packed uint8 weights, fp32 norms, uint16 fp16 caches that are
    updated in place). f64=True runs oracle_decode_step_f64 instead (every sum
    in fp64: a higher-precision measure, not the reference's arithmetic)."""
    c = ModelCfg(**{k: cfg[k] for k in ("n_layer", "d_model", "n_head", "n_kv_head", "head_dim", "d_ff", "vocab",
                                         "ctx")}, rms_eps=cfg.get("rms_eps", 1e-6),
                 rope_base=cfg.get("rope_base", 10000.0), qtype=cfg["qtype"])
    arr = (LayerPtrs * len(layers))()
    keep = []
    for i, d in enumerate(layers):
        for name, _ in LayerPtrs._fields_:
            a = d[name]
            assert a.flags["C_CONTIGUOUS"]
            keep.append(a)
            setattr(arr[i], name, a.ctypes.data)
    logits = np.empty(cfg["vocab"], np.float32)
    x = np.ascontiguousarray(x_in, np.float32)
    on = np.ascontiguousarray(out_norm, np.float32)
    fn = lib().oracle_decode_step_f64 if f64 else lib().oracle_decode_step
    rc = fn(ctypes.byref(c), arr, _p(on, _f32p), w_out.ctypes.data, _p(x, _f32p),
                                  int(pos), _p(logits, _f32p), n_threads or n_threads_default())
    if rc:
        raise RuntimeError("oracle_decode_step failed")
    return logits
