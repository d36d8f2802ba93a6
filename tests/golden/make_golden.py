"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the reference tree and the third-party `gguf`
0.19.0 Python package (the GPU hosts have neither; they only read the .npz):

    python tests/golden/make_golden.py

What each fixture pins, and with what:

* ``dequant_<TYPE>.npz`` -- packed blocks with hand-placed edge patterns
  (all-zero blocks, maximum nibbles/bits, negative and subnormal fp16 scales,
  largest 6-bit scales and mins) plus seeded random bytes, and the fp32 values
  that `gguf.quants.dequantize` (an independent decoder of the published GGUF
  block format) produces for them. The oracle and the CUDA dequantizer must
  match these bit for bit.
* ``quantize_<TYPE>.npz`` (Q4_0, Q8_0) -- seeded fp32 blocks and the bytes
  `gguf.quants.quantize` produces, pinning the oracle's seeded-weight
  generator for the two types that package can quantize.
* ``matvec_<TYPE>.npz`` -- a small seeded weight matrix, activations and
  ``y = ref_cpu_matmul_f32(gguf_dequant(W), x)``: the reference's own scalar
  matmul (src/backend/cpu_backend.cpp:24-41, compiled by oracle/build.py) on
  the independently decoded weights.
* ``kat_reference.npz`` -- the known answers of hesa-llm's own tests
  (tests/test_main.cpp:87-185: 2x3 @ 3x2 matmul, rms_norm of [3,4], silu,
  rope at positions 0 and 1), recomputed by the reference's kernels.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

SEED = 20261201


def _gguf():
    from gguf import GGMLQuantizationType as T
    from gguf import quants as GQ
    return T, GQ


def _fp16_bits(v: float) -> int:
    return int(np.array(v, dtype=np.float16).view(np.uint16))


def edge_blocks(qtype: int, rng: np.random.Generator, n_random: int) -> np.ndarray:
    bb = O.BLOCK_BYTES[qtype]
    blocks = []

    def scale_pos(b: np.ndarray, d: float, dmin: float | None = None):
        if qtype == O.Q6_K:
            b[208:210] = np.frombuffer(np.uint16(_fp16_bits(d)).tobytes(), np.uint8)
        else:
            b[0:2] = np.frombuffer(np.uint16(_fp16_bits(d)).tobytes(), np.uint8)
            if dmin is not None:
                b[2:4] = np.frombuffer(np.uint16(_fp16_bits(dmin)).tobytes(), np.uint8)

    # 1. all-zero block
    blocks.append(np.zeros(bb, np.uint8))
    # 2. all quant bits set, positive scales
    b = np.full(bb, 0xFF, np.uint8)
    scale_pos(b, 0.0123, 0.0045)
    blocks.append(b)
    # 3. all quant bits set, negative scale
    b = np.full(bb, 0xFF, np.uint8)
    scale_pos(b, -0.5, -0.25)
    blocks.append(b)
    # 4. subnormal fp16 scale(s)
    b = rng.integers(0, 256, bb, dtype=np.uint8)
    scale_pos(b, 2.0 ** -20, 3 * 2.0 ** -24)
    blocks.append(b)
    # 5. largest finite fp16 scale with small quant values
    b = np.zeros(bb, np.uint8)
    scale_pos(b, 65504.0, 1.0)
    if qtype == O.Q6_K:
        b[192:208] = 1
    elif qtype in (O.Q4_K, O.Q5_K):
        b[4:16] = 0x41
    blocks.append(b)
    # 6. alternating nibble pattern
    b = np.tile(np.array([0x5A, 0xA5], np.uint8), bb // 2 + 1)[:bb].copy()
    scale_pos(b, 1.0, 0.5)
    blocks.append(b)
    # 7.. seeded random bytes with finite, moderate scales
    for _ in range(n_random):
        b = rng.integers(0, 256, bb, dtype=np.uint8)
        scale_pos(b, float(rng.normal(0, 0.01)), float(abs(rng.normal(0, 0.01))))
        blocks.append(b)
    return np.stack(blocks)


def make_dequant(T, GQ, rng):
    for name, qt in O.QTYPES.items():
        blocks = edge_blocks(qt, rng, 26)
        expect = GQ.dequantize(blocks, T[name]).astype(np.float32).reshape(blocks.shape[0], -1)
        np.savez_compressed(os.path.join(HERE, f"dequant_{name}.npz"),
                            qtype=qt, blocks=blocks, expect=expect)


def make_quantize(T, GQ, rng):
    for name in ("Q4_0", "Q8_0"):
        w = (rng.standard_normal((24, 256), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        w[0, :] = 0.0                      # all-zero block row
        w[1, :32] = np.float32(1e-8)       # tiny values
        w[2, 5] = np.float32(-0.5)         # single dominant negative value
        blocks = GQ.quantize(w, T[name])
        np.savez_compressed(os.path.join(HERE, f"quantize_{name}.npz"),
                            qtype=O.QTYPES[name], w=w, blocks=blocks)


def make_matvec(T, GQ, rng):
    ref = O.ref_lib()
    if ref is None:
        raise SystemExit("reference CPU library unavailable: run in the container with the reference tree")
    f32p = ctypes.POINTER(ctypes.c_float)
    for name, qt in O.QTYPES.items():
        n_out, k, B = 24, 768, 3
        w = O.gaussian((n_out, k), 0.02, SEED + qt)
        blocks = O.quantize(qt, w)
        deq = GQ.dequantize(blocks, T[name]).astype(np.float32).reshape(n_out, k)
        x = O.gaussian((B, k), 1.0, SEED + 100 + qt)
        y = np.empty((B, n_out), np.float32)
        for b in range(B):
            xb = np.ascontiguousarray(x[b])
            yb = np.empty(n_out, np.float32)
            ref.ref_cpu_matmul_f32(deq.ctypes.data_as(f32p), xb.ctypes.data_as(f32p),
                                   yb.ctypes.data_as(f32p), n_out, 1, k, ctypes.c_float(0.75))
            y[b] = yb
        np.savez_compressed(os.path.join(HERE, f"matvec_{name}.npz"),
                            qtype=qt, blocks=blocks, x=x, scale=np.float32(0.75), y=y)


def make_kat():
    ref = O.ref_lib()
    f32p = ctypes.POINTER(ctypes.c_float)
    a = np.array([1, 2, 3, 4, 5, 6], np.float32)
    b = np.array([7, 8, 9, 10, 11, 12], np.float32)
    c = np.empty(4, np.float32)
    ref.ref_cpu_matmul_f32(a.ctypes.data_as(f32p), b.ctypes.data_as(f32p), c.ctypes.data_as(f32p),
                           2, 2, 3, ctypes.c_float(1.0))
    rin = np.array([3, 4], np.float32)
    rw = np.ones(2, np.float32)
    rout = np.empty(2, np.float32)
    ref.ref_cpu_rms_norm_f32(rin.ctypes.data_as(f32p), rw.ctypes.data_as(f32p),
                             rout.ctypes.data_as(f32p), 1, 2, ctypes.c_float(1e-6))
    sin = np.array([0, 1, -1], np.float32)
    sout = np.empty(3, np.float32)
    ref.ref_cpu_silu_f32(sin.ctypes.data_as(f32p), sout.ctypes.data_as(f32p), 3)
    pos = (ctypes.c_int32 * 1)()
    r0 = np.array([1, 2, 3, 4], np.float32)
    pos[0] = 0
    ref.ref_cpu_rope_f32(r0.ctypes.data_as(f32p), pos, 1, 1, 4, ctypes.c_float(10000.0))
    r1 = np.array([1, 0, 0, 1], np.float32)
    pos[0] = 1
    ref.ref_cpu_rope_f32(r1.ctypes.data_as(f32p), pos, 1, 1, 4, ctypes.c_float(10000.0))
    # a longer rope case: 4 heads x 128 at position 2047
    rl = O.gaussian((4 * 128,), 1.0, SEED + 7)
    rl_out = rl.copy()
    pos[0] = 2047
    ref.ref_cpu_rope_f32(rl_out.ctypes.data_as(f32p), pos, 1, 4, 128, ctypes.c_float(10000.0))
    nl = O.gaussian((4096,), 1.0, SEED + 8)
    nw = O.gaussian((4096,), 1.0, SEED + 9)
    nl_out = np.empty_like(nl)
    ref.ref_cpu_rms_norm_f32(nl.ctypes.data_as(f32p), nw.ctypes.data_as(f32p),
                             nl_out.ctypes.data_as(f32p), 1, 4096, ctypes.c_float(1e-6))
    np.savez_compressed(os.path.join(HERE, "kat_reference.npz"),
                        matmul=c, rms_in=rin, rms_out=rout, silu_in=sin, silu_out=sout,
                        rope_pos0=r0, rope_pos1=r1, rope_long_in=rl, rope_long_out=rl_out,
                        rms_long_in=nl, rms_long_w=nw, rms_long_out=nl_out)


def main():
    T, GQ = _gguf()
    rng = np.random.default_rng(SEED)
    make_dequant(T, GQ, rng)
    make_quantize(T, GQ, rng)
    make_matvec(T, GQ, rng)
    make_kat()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
