"""Python binding of the hesa-b200 C ABI (include/hesa_cuda.h) over ctypes.

This is the host-side mirror of the reference's operator interface for the
hot path: ``qmatvec`` is ``hesa::Backend::matmul`` (include/hesa/backend.hpp:
43-44) for a quantized weight, with the same argument meaning (W [n_out, k],
activations [batch, k], out = scale * W @ x) and the same error codes
(``hesa::Error``, include/hesa/result.hpp:14-30), raised as ``HesaError``.

PyTorch is only plumbing here: it owns device memory and streams. Every
computation runs in ``libhesa_cuda.so``; if that library cannot be built or
loaded, every call raises -- there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os

import hesa_build as _build

Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 8, 12, 13, 14
QTYPES = {"Q4_0": Q4_0, "Q8_0": Q8_0, "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210}

ERRORS = {0: "SUCCESS", 1: "OUT_OF_MEMORY", 2: "INVALID_ARGUMENT", 3: "BACKEND_NOT_AVAILABLE",
          6: "SHAPE_MISMATCH", 8: "INVALID_FORMAT", 9: "CUDA_ERROR", 14: "INTERNAL_ERROR"}

# (name, restype, argtypes) of every function include/hesa_cuda.h declares
_vp, _i64, _sz, _int, _f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_int, ctypes.c_float


class Model(ctypes.Structure):
    """hesa_cuda_model (include/hesa_cuda.h)."""
    _fields_ = [("n_layer", ctypes.c_int32), ("d_model", ctypes.c_int32), ("n_head", ctypes.c_int32),
                ("n_kv_head", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("d_ff", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("ctx", ctypes.c_int32), ("rms_eps", ctypes.c_float),
                ("rope_base", ctypes.c_float), ("qtype", ctypes.c_int32)]


class Layer(ctypes.Structure):
    """hesa_cuda_layer (include/hesa_cuda.h): device pointers of one layer."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm",
                                              "ffn_norm", "k_cache", "v_cache")]

SIGNATURES = [
    ("hesa_cuda_version", ctypes.c_char_p, []),
    ("hesa_cuda_row_bytes", _sz, [_int, _i64]),
    ("hesa_cuda_qmatvec_workspace_size", _sz, [_int, _i64, _i64, _i64]),
    ("hesa_cuda_qmatvec", _int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _f, _vp, _sz, _vp]),
    ("hesa_cuda_qmatvec_noalloc", _int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _f, _vp]),
    ("hesa_cuda_dequantize", _int, [_int, _vp, _i64, _i64, _vp, _i64, _vp]),
    ("hesa_cuda_quantize", _int, [_int, _vp, _i64, _i64, _i64, _vp, _vp]),
    ("hesa_cuda_device_status", _int, [_vp, ctypes.POINTER(_int)]),
    ("hesa_cuda_clear_device_status", _int, [_vp]),
    ("hesa_cuda_last_error", ctypes.c_char_p, []),
    ("hesa_cuda_matmul_f32", _int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _f, _vp]),
    ("hesa_cuda_rms_norm", _int, [_vp, _vp, _vp, _i64, _i64, _f, _vp]),
    ("hesa_cuda_silu_mul", _int, [_vp, _vp, _vp, _i64, _vp]),
    ("hesa_cuda_add", _int, [_vp, _vp, _vp, _i64, _vp]),
    ("hesa_cuda_mul", _int, [_vp, _vp, _vp, _i64, _vp]),
    ("hesa_cuda_softmax", _int, [_vp, _vp, _i64, _i64, _vp]),
    ("hesa_cuda_rope_table", _int, [_vp, ctypes.c_int32, _i64, _f]),
    ("hesa_cuda_rope", _int, [_vp, _i64, _i64, _vp, ctypes.c_int32, _vp, ctypes.c_int32, _vp]),
    ("hesa_cuda_kv_store", _int, [_vp, _vp, _vp, _vp, _i64, _i64, _vp, ctypes.c_int32, _vp]),
    ("hesa_cuda_attention_workspace_size", _sz, [_i64, _i64, _i64]),
    ("hesa_cuda_attention", _int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, ctypes.c_int32, _vp, _sz,
                                   _vp]),
    ("hesa_cuda_decode_workspace_size", _sz, [ctypes.POINTER(Model)]),
    ("hesa_cuda_embed", _int, [_int, _vp, _i64, _i64, _vp, _vp, _vp]),
    ("hesa_cuda_decode_step", _int, [ctypes.POINTER(Model), ctypes.POINTER(Layer), _vp, _vp, _vp, ctypes.c_int32,
                                     _vp, _vp, _vp, _vp, _sz, _vp]),
    ("hesa_cuda_peer_alloc", _int, [_sz, ctypes.POINTER(_vp), _vp]),
    ("hesa_cuda_peer_free", _int, [_vp]),
    ("hesa_cuda_peer_open", _int, [_vp, ctypes.POINTER(_vp)]),
    ("hesa_cuda_peer_close", _int, [_vp]),
    ("hesa_cuda_qmatvec_gather", _int, [_int, _vp, _i64, _i64, _vp, _f, ctypes.POINTER(_vp), _int, _vp, _vp]),
    ("hesa_cuda_peer_barrier", _int, [ctypes.POINTER(_vp), _int, _int, _vp, _vp]),
    ("hesa_cuda_gather_tagged_workspace_size", _sz, [_int, _i64, _i64]),
    ("hesa_cuda_qmatvec_gather_tagged", _int, [_int, _vp, _i64, _i64, _vp, _f, ctypes.POINTER(_vp), _i64, _int,
                                               _vp, _vp, _sz, _vp]),
    ("hesa_cuda_peer_collect", _int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    ("hesa_cuda_set_peer_wait_limit_us", _int, [ctypes.c_uint32]),
    ("hesa_cuda_decode_step_sharded", _int, [ctypes.POINTER(Model), _vp, ctypes.POINTER(Layer), _vp, _vp, _vp,
                                             ctypes.c_int32, _vp, _vp, _vp, _vp, _sz, _vp]),
]


class Shard(ctypes.Structure):
    """hesa_cuda_shard (include/hesa_cuda.h): one rank of a head-sharded decode."""
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("a_peers", ctypes.c_void_p),
                ("gu_peers", ctypes.c_void_p), ("logits_peers", ctypes.c_void_p), ("token_count", ctypes.c_void_p)]

    def __init__(self, rank, world, a, gu, logits, token_count):
        super().__init__(rank, world, ctypes.cast(a, ctypes.c_void_p), ctypes.cast(gu, ctypes.c_void_p),
                         ctypes.cast(logits, ctypes.c_void_p), token_count)


class HesaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)} ({code}): {msg}")
        self.code = code


_lib = None


def library_path() -> str:
    return _build.CUDA_SO


def lib() -> ctypes.CDLL:
    """Load libhesa_cuda.so, building it first if it is missing or stale."""
    global _lib
    if _lib is None:
        path = _build.build_cuda()
        L = ctypes.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise HesaError(rc, lib().hesa_cuda_last_error().decode())


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream or None
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


def row_bytes(qtype: int, k: int) -> int:
    return int(lib().hesa_cuda_row_bytes(qtype, k))


def workspace_bytes(qtype: int, n_out: int, k: int, batch: int = 1) -> int:
    return int(lib().hesa_cuda_qmatvec_workspace_size(qtype, n_out, k, batch))


def make_workspace(qtype: int, n_out: int, k: int, batch: int = 1, device=None):
    """A zero-filled device workspace of the size the matvec asks for."""
    import torch
    nbytes = max(16, workspace_bytes(qtype, n_out, k, batch))
    return torch.zeros(nbytes, dtype=torch.uint8, device=device or "cuda")


def qmatvec(qtype: int, w, x, y=None, scale: float = 1.0, workspace=None, stream=None, k: int | None = None):
    """y = scale * W @ x for packed W [n_out, row_bytes] (uint8, CUDA) and fp32
    x [k] or [batch, k]; returns y [n_out] or [batch, n_out]."""
    import torch
    squeeze = x.dim() == 1
    x2 = x.unsqueeze(0) if squeeze else x
    batch, kk = x2.shape
    k = k or kk
    n_out = w.shape[0]
    if y is None:
        y = torch.empty((batch, n_out), dtype=torch.float32, device=x.device)
    y2 = y.unsqueeze(0) if y.dim() == 1 else y
    if workspace is None:
        workspace = make_workspace(qtype, n_out, k, batch, device=x.device)
    rc = lib().hesa_cuda_qmatvec(qtype, w.data_ptr(), n_out, k, x2.data_ptr(), x2.stride(0), batch,
                                 y2.data_ptr(), y2.stride(0), float(scale), workspace.data_ptr(),
                                 workspace.numel(), _stream_handle(stream))
    _check(rc)
    return y2[0] if squeeze else y2


def dequantize(qtype: int, w, k: int, out=None, stream=None):
    import torch
    n_rows = w.shape[0]
    if out is None:
        out = torch.empty((n_rows, k), dtype=torch.float32, device=w.device)
    _check(lib().hesa_cuda_dequantize(qtype, w.data_ptr(), n_rows, k, out.data_ptr(), out.stride(0),
                                      _stream_handle(stream)))
    return out


def quantize(qtype: int, x, out=None, stream=None):
    """Packed GGUF rows [n_rows, row_bytes] (uint8, CUDA) of fp32 x [n_rows, k]
    (CUDA), deterministic round-to-nearest (hesa_cuda_quantize)."""
    import torch
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    n_rows, k = x2.shape
    if x2.stride(1) != 1:
        raise ValueError("rows of x must be contiguous")
    rb = row_bytes(qtype, k)
    if rb == 0:
        raise HesaError(6, f"k={k} is not a multiple of the block size of qtype {qtype}")
    if out is None:
        out = torch.empty((n_rows, rb), dtype=torch.uint8, device=x.device)
    _check(lib().hesa_cuda_quantize(qtype, x2.data_ptr(), n_rows, k, x2.stride(0), out.data_ptr(),
                                    _stream_handle(stream)))
    return out


# ---- row-sharded matvec with the all-gather fused in (hesa_cuda_qmatvec_gather) ----

def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """A zero-filled device allocation shared with the other ranks of the node:
    (device pointer, 64-byte CUDA IPC handle)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _check(lib().hesa_cuda_peer_alloc(nbytes, ctypes.byref(ptr), handle))
    return ptr.value, handle.raw


def peer_free(ptr: int) -> None:
    _check(lib().hesa_cuda_peer_free(ptr))


def peer_open(handle: bytes) -> int:
    """Map another rank's peer_alloc allocation into this process."""
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), 64)
    _check(lib().hesa_cuda_peer_open(buf, ctypes.byref(ptr)))
    return ptr.value


def peer_close(ptr: int) -> None:
    _check(lib().hesa_cuda_peer_close(ptr))


def qmatvec_gather(qtype: int, w, x, y_peers, world: int, epoch: int, scale: float = 1.0, stream=None):
    """This rank's rows of y = scale * W x (w: its packed rows [n_rows, row_bytes],
    x [k]) stored into every rank's gathered buffer: y_peers lists 2 * world
    device addresses (parity-major) of this shard's first row in each rank's
    buffer; epoch is the device address of this rank's barrier count."""
    n_rows, k = w.shape[0], x.shape[-1]
    arr = (ctypes.c_void_p * (2 * world))(*y_peers)
    _check(lib().hesa_cuda_qmatvec_gather(qtype, w.data_ptr(), n_rows, k, x.data_ptr(), float(scale), arr, world,
                                          epoch, _stream_handle(stream)))


def gather_tagged_workspace(qtype: int, n_rows: int, k: int, device=None):
    """The workspace qmatvec_gather_tagged needs for this shape (None when the
    row-strip kernel takes it and none is needed)."""
    import torch
    nbytes = lib().hesa_cuda_gather_tagged_workspace_size(qtype, n_rows, k)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device or "cuda") if nbytes else None


def qmatvec_gather_tagged(qtype: int, w, x, y_peers, row0: int, world: int, sync: int, scale: float = 1.0,
                          workspace=None, stream=None):
    """As qmatvec_gather, every row stored as a tagged 64-bit word: row i is
    element row0 + i of the gathered vector; y_peers lists 2 * world device
    addresses (parity-major) of word 0 of each rank's gathered buffers; sync
    is the device address of this rank's [step count, ticket] pair. The step
    ends with peer_collect. Rows longer than the strip kernel takes need
    `workspace` (gather_tagged_workspace)."""
    n_rows, k = w.shape[0], x.shape[-1]
    if workspace is None and lib().hesa_cuda_gather_tagged_workspace_size(qtype, n_rows, k):
        workspace = gather_tagged_workspace(qtype, n_rows, k, device=x.device)
    arr = (ctypes.c_void_p * (2 * world))(*y_peers)
    _check(lib().hesa_cuda_qmatvec_gather_tagged(qtype, w.data_ptr(), n_rows, k, x.data_ptr(), float(scale), arr,
                                                 row0, world, sync,
                                                 workspace.data_ptr() if workspace is not None else None,
                                                 workspace.numel() if workspace is not None else 0,
                                                 _stream_handle(stream)))


def peer_collect(words: int, n: int, parity_stride: int, out, sync: int, stream=None) -> None:
    """Wait for this step's n tagged elements in this rank's buffer (device
    address of word 0 `words`, parity 1 `parity_stride` words further, a
    multiple of 256), unpack them into out (fp32 device tensor of n values)
    and advance the step count."""
    import torch
    if out.numel() < n or out.dtype != torch.float32:
        raise ValueError("out must hold n fp32 values")
    _check(lib().hesa_cuda_peer_collect(words, n, parity_stride, out.data_ptr(), sync, _stream_handle(stream)))


def peer_barrier(flags, rank: int, world: int, epoch: int, stream=None) -> None:
    arr = (ctypes.c_void_p * world)(*flags)
    _check(lib().hesa_cuda_peer_barrier(arr, rank, world, epoch, _stream_handle(stream)))


def set_peer_wait_limit(seconds: float) -> None:
    """How long each peer barrier waits for the other ranks before it gives up
    and records device status 4 (0 restores the default, 2 s)."""
    _check(lib().hesa_cuda_set_peer_wait_limit_us(int(round(seconds * 1e6))))


def device_view(ptr: int, numel: int, device=None, dtype: str = "<f4"):
    """A torch tensor over raw device memory (no copy), through the CUDA array
    interface."""
    import torch

    class _View:
        __cuda_array_interface__ = {"shape": (numel,), "typestr": dtype, "data": (ptr, False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_View(), device=device or "cuda")


def device_status(stream=None) -> int:
    v = ctypes.c_int(0)
    _check(lib().hesa_cuda_device_status(_stream_handle(stream), ctypes.byref(v)))
    return v.value


def clear_device_status(stream=None) -> None:
    _check(lib().hesa_cuda_clear_device_status(_stream_handle(stream)))


def loaded_library_files() -> list[str]:
    """Shared objects of this package mapped into the current process."""
    out = []
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                p = line.split()[-1]
                if p.endswith(".so") and os.path.dirname(p) == os.path.dirname(library_path()):
                    out.append(p)
    except OSError:
        pass
    return sorted(set(out))


# --------------------------------------------------------------------------
# decode-step helpers (device tensors in, device tensors out)
# --------------------------------------------------------------------------

def _ptr(t):
    return None if t is None else t.data_ptr()


def matmul_f32(a, x, y=None, scale: float = 1.0, stream=None):
    import torch
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    batch, k = x2.shape
    n_out = a.shape[0]
    if y is None:
        y = torch.empty((batch, n_out), dtype=torch.float32, device=x.device)
    y2 = y.unsqueeze(0) if y.dim() == 1 else y
    _check(lib().hesa_cuda_matmul_f32(a.data_ptr(), n_out, k, x2.data_ptr(), x2.stride(0), batch, y2.data_ptr(),
                                      y2.stride(0), float(scale), _stream_handle(stream)))
    return y2[0] if x.dim() == 1 else y2


def rms_norm(x, w, eps: float = 1e-6, out=None, stream=None):
    import torch
    out = torch.empty_like(x) if out is None else out
    n = x.shape[-1]
    _check(lib().hesa_cuda_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), x.numel() // n, n, float(eps),
                                    _stream_handle(stream)))
    return out


def silu_mul(g, u=None, out=None, stream=None):
    import torch
    out = torch.empty_like(g) if out is None else out
    _check(lib().hesa_cuda_silu_mul(g.data_ptr(), _ptr(u), out.data_ptr(), g.numel(), _stream_handle(stream)))
    return out


def add(a, b, out=None, stream=None):
    import torch
    out = torch.empty_like(a) if out is None else out
    _check(lib().hesa_cuda_add(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream_handle(stream)))
    return out


def mul(a, b, out=None, stream=None):
    import torch
    out = torch.empty_like(a) if out is None else out
    _check(lib().hesa_cuda_mul(a.data_ptr(), b.data_ptr(), out.data_ptr(), a.numel(), _stream_handle(stream)))
    return out


def softmax(x, out=None, stream=None):
    import torch
    out = torch.empty_like(x) if out is None else out
    n = x.shape[-1]
    _check(lib().hesa_cuda_softmax(x.data_ptr(), out.data_ptr(), x.numel() // n, n, _stream_handle(stream)))
    return out


def rope_table(n_pos: int, head_dim: int, base: float = 10000.0):
    """Host-computed rotate-half angle table [n_pos, head_dim] (numpy)."""
    import numpy as np
    t = np.empty((n_pos, head_dim), dtype=np.float32)
    _check(lib().hesa_cuda_rope_table(t.ctypes.data, n_pos, head_dim, float(base)))
    return t


def rope(x, n_heads: int, head_dim: int, table, pos=None, pos_dev=None, stream=None):
    _check(lib().hesa_cuda_rope(x.data_ptr(), n_heads, head_dim, table.data_ptr(), table.shape[0],
                                _ptr(pos_dev), int(pos or 0), _stream_handle(stream)))
    return x


def kv_store(k, v, k_cache, v_cache, ctx: int, pos=None, pos_dev=None, stream=None):
    _check(lib().hesa_cuda_kv_store(k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k.numel(),
                                    ctx, _ptr(pos_dev), int(pos or 0), _stream_handle(stream)))


def attention_workspace(n_head: int, head_dim: int, ctx: int, device=None):
    import torch
    nb = int(lib().hesa_cuda_attention_workspace_size(n_head, head_dim, ctx))
    return torch.zeros(max(nb, 16), dtype=torch.uint8, device=device or "cuda")


def attention(q, k_cache, v_cache, n_head: int, n_kv_head: int, head_dim: int, ctx: int, pos=None, pos_dev=None,
              workspace=None, out=None, stream=None):
    import torch
    out = torch.empty_like(q) if out is None else out
    if workspace is None:
        workspace = attention_workspace(n_head, head_dim, ctx, device=q.device)
    _check(lib().hesa_cuda_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), n_head,
                                     n_kv_head, head_dim, ctx, _ptr(pos_dev), int(pos or 0), workspace.data_ptr(),
                                     workspace.numel(), _stream_handle(stream)))
    return out


# ---------------------------------------------------------------------------
# decode step
# ---------------------------------------------------------------------------

def decode_workspace(model: Model, device=None):
    """Zero-filled workspace of hesa_cuda_decode_step (uint8, 256-byte aligned)."""
    import torch
    nb = int(lib().hesa_cuda_decode_workspace_size(ctypes.byref(model)))
    if nb == 0:
        raise HesaError(6, "bad model shape")
    return torch.zeros(nb, dtype=torch.uint8, device=device or "cuda")


def embed(qtype: int, w_emb, d_model: int, token_dev, out=None, stream=None):
    import torch
    out = torch.empty(d_model, dtype=torch.float32, device=w_emb.device) if out is None else out
    _check(lib().hesa_cuda_embed(qtype, w_emb.data_ptr(), w_emb.shape[0], d_model, token_dev.data_ptr(),
                                 out.data_ptr(), _stream_handle(stream)))
    return out


def decode_step(model: Model, layers, out_norm, w_out, rope_table, x_embed, pos_dev, logits, workspace,
                stream=None):
    """One token through the decoder (hesa_cuda_decode_step). `layers` is a
    ctypes array of Layer (see make_layers)."""
    _check(lib().hesa_cuda_decode_step(ctypes.byref(model), layers, out_norm.data_ptr(), w_out.data_ptr(),
                                       rope_table.data_ptr(), rope_table.shape[0], x_embed.data_ptr(),
                                       pos_dev.data_ptr(), logits.data_ptr(), workspace.data_ptr(),
                                       workspace.numel(), _stream_handle(stream)))
    return logits


def decode_step_sharded(model: Model, shard, layers, out_norm, w_out, rope_table, x_embed, pos_dev, logits,
                        workspace, stream=None):
    """This rank's part of one token of a head-sharded decode
    (hesa_cuda_decode_step_sharded); every rank gets all the logits."""
    _check(lib().hesa_cuda_decode_step_sharded(ctypes.byref(model), ctypes.byref(shard), layers, out_norm.data_ptr(),
                                               w_out.data_ptr(), rope_table.data_ptr(), rope_table.shape[0],
                                               x_embed.data_ptr(), pos_dev.data_ptr(), logits.data_ptr(),
                                               workspace.data_ptr(), workspace.numel(), _stream_handle(stream)))


def make_layers(per_layer):
    """ctypes array of Layer from a list of dicts of CUDA tensors with the
    keys of Layer's fields."""
    arr = (Layer * len(per_layer))()
    for i, d in enumerate(per_layer):
        for name, _ in Layer._fields_:
            setattr(arr[i], name, d[name].data_ptr())
    return arr
