"""GPU parity of the decode-step helper kernels (C ABI) against the oracle's
restatement of hesa-llm's CPU kernels and the reference's own known answers."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REL_L2_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def T():
    import torch
    assert torch.cuda.is_available()
    import hesa_cuda
    hesa_cuda.lib()
    return torch


def dev(T, a):
    return T.from_numpy(np.ascontiguousarray(a)).cuda()


def test_reference_kat_matmul_f32(T):
    """tests/test_main.cpp:87-108: [1,2,3;4,5,6] @ [7,8;9,10;11,12]."""
    import hesa_cuda as H
    a = dev(T, np.array([[1, 2, 3], [4, 5, 6]], np.float32))
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    y = H.matmul_f32(a, dev(T, b.T.copy())).cpu().numpy()   # y[j, i] = sum_k a[i,k] b[k,j]
    np.testing.assert_allclose(y.T, [[58, 64], [139, 154]], atol=1e-3)


def test_rms_norm_kat_and_long_row(T):
    import hesa_cuda as H
    kat = np.load(os.path.join(GOLDEN, "kat_reference.npz"))
    out = H.rms_norm(dev(T, kat["rms_in"]), dev(T, np.ones(2, np.float32))).cpu().numpy()
    np.testing.assert_allclose(out, kat["rms_out"], rtol=1e-6)
    out = H.rms_norm(dev(T, kat["rms_long_in"]), dev(T, kat["rms_long_w"])).cpu().numpy()
    assert rel_l2(out, kat["rms_long_out"]) <= REL_L2_TOL


def test_silu_mul_add_mul_softmax(T):
    import hesa_cuda as H
    kat = np.load(os.path.join(GOLDEN, "kat_reference.npz"))
    s = H.silu_mul(dev(T, kat["silu_in"])).cpu().numpy()
    np.testing.assert_allclose(s, kat["silu_out"], rtol=1e-6, atol=1e-7)
    g = O.gaussian((11008,), 2.0, 1)
    u = O.gaussian((11008,), 1.0, 2)
    got = H.silu_mul(dev(T, g), dev(T, u)).cpu().numpy()
    assert rel_l2(got, O.silu_mul(g, u)) <= REL_L2_TOL
    np.testing.assert_array_equal(H.add(dev(T, g), dev(T, u)).cpu().numpy(), g + u)
    np.testing.assert_array_equal(H.mul(dev(T, g), dev(T, u)).cpu().numpy(), g * u)
    x = O.gaussian((3, 1000), 3.0, 3)
    sm = H.softmax(dev(T, x)).cpu().numpy()
    e = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    assert rel_l2(sm, e / e.sum(axis=1, keepdims=True)) <= REL_L2_TOL


def test_rope_table_and_kernel_bit_exact(T):
    """The host table uses the reference formulas; rope then matches the
    reference's compiled cpu_rope_f32 bit for bit (tests/golden)."""
    import hesa_cuda as H
    kat = np.load(os.path.join(GOLDEN, "kat_reference.npz"))
    table = H.rope_table(2048, 128)
    c, s = O.rope_table(2047, 128)
    assert np.array_equal(table[2047, :64], c) and np.array_equal(table[2047, 64:], s)
    x = dev(T, kat["rope_long_in"])
    H.rope(x, 4, 128, dev(T, table), pos=2047)
    assert np.array_equal(x.cpu().numpy(), kat["rope_long_out"])
    t4 = H.rope_table(2, 4)
    x = dev(T, np.array([1, 0, 0, 1], np.float32))
    pos = dev(T, np.array([1], np.int32))
    H.rope(x, 1, 4, dev(T, t4), pos_dev=pos)
    assert np.array_equal(x.cpu().numpy(), kat["rope_pos1"])


def test_kv_store_ring_and_fp16_rounding(T):
    import hesa_cuda as H
    ctx, row = 16, 2 * 64
    kc = T.zeros((ctx, row), dtype=T.float16, device="cuda")
    vc = T.zeros_like(kc)
    k = O.gaussian((row,), 1.0, 4)
    v = O.gaussian((row,), 1.0, 5)
    H.kv_store(dev(T, k), dev(T, v), kc, vc, ctx, pos=21)   # slot 5
    kn = kc.cpu().numpy().view(np.uint16)
    assert np.array_equal(kn[5], O.fp32_to_fp16_bits(k))
    assert np.array_equal(vc.cpu().numpy().view(np.uint16)[5], O.fp32_to_fp16_bits(v))
    assert not kn[[0, 4, 6]].any()


@pytest.mark.parametrize("n_head,n_kv,hd,ctx,pos", [
    (32, 32, 128, 2048, 2047),   # 7B shape, full context
    (32, 32, 128, 2048, 100),    # partly filled ring
    (64, 8, 128, 512, 700),      # GQA, wrapped ring
    (8, 2, 64, 37, 36),
    (4, 4, 256, 300, 0),         # first token
])
def test_attention_matches_oracle(T, n_head, n_kv, hd, ctx, pos):
    import hesa_cuda as H
    rng = np.random.default_rng(n_head + ctx + pos)
    q = rng.standard_normal(n_head * hd).astype(np.float32)
    kc = rng.standard_normal((ctx, n_kv * hd)).astype(np.float16)
    vc = rng.standard_normal((ctx, n_kv * hd)).astype(np.float16)
    n_ctx = min(pos + 1, ctx)
    ws = H.attention_workspace(n_head, hd, ctx)
    out = H.attention(dev(T, q), dev(T, kc), dev(T, vc), n_head, n_kv, hd, ctx, pos=pos, workspace=ws)
    out2 = H.attention(dev(T, q), dev(T, kc), dev(T, vc), n_head, n_kv, hd, ctx,
                       pos_dev=dev(T, np.array([pos], np.int32)), workspace=ws)
    ref = O.attention_f16kv(q, kc.view(np.uint16), vc.view(np.uint16), n_head, n_kv, hd, n_ctx)
    assert rel_l2(out.cpu().numpy(), ref) <= REL_L2_TOL
    assert T.equal(out, out2)
