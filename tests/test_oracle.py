"""CPU tests: the oracle against the committed golden fixtures and the
reference's own known answers. These pin the oracle before any GPU result is
compared with it."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_dequant_matches_independent_decoder(name):
    g = _load(f"dequant_{name}.npz")
    qt = int(g["qtype"])
    blocks = g["blocks"]
    k = O.BLOCK_ELEMS[qt]
    got = O.dequantize(qt, blocks, k)
    exp = g["expect"].reshape(blocks.shape[0], k)
    # bit-exact, including signed zeros
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("name", ["Q4_0", "Q8_0"])
def test_quantizer_matches_published_rounding(name):
    g = _load(f"quantize_{name}.npz")
    got = O.quantize(int(g["qtype"]), g["w"])
    assert np.array_equal(got, g["blocks"])


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_qmatvec_matches_reference_matmul(name):
    """oracle qmatvec == the reference's cpu_matmul_f32 on independently
    decoded weights, bit for bit (same k order, separate mul and add)."""
    g = _load(f"matvec_{name}.npz")
    y = O.qmatvec(int(g["qtype"]), g["blocks"], g["x"], scale=float(g["scale"]))
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_qmatvec_thread_count_independent(threads):
    g = _load("matvec_Q4_K.npz")
    y = O.qmatvec(int(g["qtype"]), g["blocks"], g["x"], scale=float(g["scale"]), n_threads=threads)
    assert np.array_equal(y, g["y"])


def test_reference_known_answers():
    """hesa-llm tests/test_main.cpp:87-148 known answers, through the oracle."""
    kat = _load("kat_reference.npz")
    np.testing.assert_allclose(kat["matmul"], [58, 64, 139, 154], atol=1e-3)
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    np.testing.assert_allclose(a @ b, kat["matmul"].reshape(2, 2))
    out = O.rms_norm(kat["rms_in"], np.ones(2, np.float32))
    assert np.array_equal(out, kat["rms_out"])
    rms = np.sqrt(np.float32(12.5))
    np.testing.assert_allclose(out, [3 / rms, 4 / rms], atol=1e-4)
    s = O.silu_mul(kat["silu_in"], np.ones(3, np.float32))
    assert np.array_equal(s, kat["silu_out"])
    np.testing.assert_allclose(s[1], 1 / (1 + np.exp(-1)), atol=1e-4)


def test_rope_matches_reference_kernel():
    """Rotate-half rope (cpu_backend.cpp:98-120), bit-exact with the
    reference's compiled kernel. At position 0 it is the identity."""
    kat = _load("kat_reference.npz")
    assert np.array_equal(O.rope(np.array([1, 2, 3, 4], np.float32), 0, 1, 4), kat["rope_pos0"])
    assert np.array_equal(O.rope(np.array([1, 0, 0, 1], np.float32), 1, 1, 4), kat["rope_pos1"])
    assert np.array_equal(O.rope(kat["rope_long_in"], 2047, 4, 128), kat["rope_long_out"])


def test_rms_norm_long_row_matches_reference_kernel():
    kat = _load("kat_reference.npz")
    got = O.rms_norm(kat["rms_long_in"], kat["rms_long_w"])
    assert np.array_equal(got, kat["rms_long_out"])


def test_fp16_roundtrip_and_rounding():
    L = O.lib()
    for bits in [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0xFBFF, 0x7C00]:
        f = L.oracle_fp16_to_fp32(bits)
        assert L.oracle_fp32_to_fp16(f) == bits
    vals = np.array([0.1, -3.3e-5, 65519.0, 65520.0, 1e-8, 2.0 ** -25, 3 * 2.0 ** -26, 1.00048828125],
                    np.float32)
    with np.errstate(over="ignore"):  # 65520 rounds to +inf in fp16, as intended
        expect = vals.astype(np.float16).view(np.uint16)
    for v, e in zip(vals, expect):
        assert L.oracle_fp32_to_fp16(float(v)) == int(e)


def test_row_bytes_match_reference_block_sizes():
    """gguf_loader.cpp:26-35: 18 B/32, 34 B/32, 144/176/210 B per 256."""
    assert O.row_bytes(O.Q4_0, 4096) == 128 * 18
    assert O.row_bytes(O.Q8_0, 11008) == 344 * 34
    assert O.row_bytes(O.Q4_K, 11008) == 43 * 144
    assert O.row_bytes(O.Q5_K, 4096) == 16 * 176
    assert O.row_bytes(O.Q6_K, 11008) == 43 * 210


def test_quantize_dequantize_error_is_small():
    w = O.gaussian((32, 1024), 0.02, 5)
    for qt, tol in [(O.Q4_0, 0.12), (O.Q8_0, 0.01), (O.Q4_K, 0.12), (O.Q5_K, 0.06), (O.Q6_K, 0.03)]:
        d = O.dequantize(qt, O.quantize(qt, w), 1024)
        assert np.linalg.norm(d - w) / np.linalg.norm(w) < tol


def test_attention_matches_numpy_fp64():
    rng = np.random.default_rng(3)
    n_head, n_kv, hd, ctx = 8, 2, 64, 37
    q = rng.standard_normal(n_head * hd).astype(np.float32)
    kc = rng.standard_normal((ctx, n_kv, hd)).astype(np.float16)
    vc = rng.standard_normal((ctx, n_kv, hd)).astype(np.float16)
    out = O.attention_f16kv(q, kc.view(np.uint16), vc.view(np.uint16), n_head, n_kv, hd, ctx)
    qq = q.reshape(n_head, hd).astype(np.float64)
    ref = np.empty((n_head, hd))
    for h in range(n_head):
        kv = h // (n_head // n_kv)
        s = kc[:, kv, :].astype(np.float64) @ qq[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        ref[h] = p @ vc[:, kv, :].astype(np.float64)
    np.testing.assert_allclose(out.reshape(n_head, hd), ref, rtol=1e-4, atol=1e-5)
