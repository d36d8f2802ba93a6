"""The decode step at the exact widths of the 7B-shaped Q4_K model the
benchmark quotes tokens/s on (d_model 4096, 32 heads x 128, FFN 11008 SwiGLU,
vocab 32000, RMSNorm eps 1e-6, RoPE base 10000, a 2048-slot fp16 KV ring),
decoding at position 2047 so attention spans the whole ring, against the
oracle's decode step (restating src/backend/cpu_backend.cpp:72-120,225-294).

At these widths the step takes code paths the small-model tests do not: the
SwiGLU input of the down projection at k = 11008 (43 units, a second staging
batch), the RMSNorm prologue at k = 4096, the 16-split attention combine and
the 32000-row LM head. The weights come from the GPU quantizer, which is
byte-identical to the oracle's (tests/test_quantize_gpu.py), and are copied
to the host for the oracle, so set-up takes seconds.

Bars: logits within rel-L2 1e-5 of the oracle at 2 layers. At 32 layers the
oracle's own fp32 rounding (the reference's arithmetic: sequential fp32 sums)
is ~1.6e-5 from the exact logits, measured with the oracle's fp64-accumulating
decode step; there the kernels must be within 1e-5 of that exact result and no
further from it than the oracle (measured on B200: 9.1e-6 against the
oracle's 1.59e-5). The KV slot the step writes within one fp16 rounding of the
oracle's and every other slot untouched."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CFG_7B = dict(n_layer=2, d_model=4096, n_head=32, n_kv_head=32, head_dim=128, d_ff=11008, vocab=32000, ctx=2048,
              rms_eps=1e-6, rope_base=10000.0, qtype=O.Q4_K)
POS = 2047


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def build(cfg, seed):
    """Device tensors (Q|K|V and gate|up rows joined, as the benchmark lays
    them out) and host copies of the same bytes for the oracle."""
    import torch
    import hesa_cuda as H
    qt = cfg["qtype"]
    D, HD = cfg["d_model"], cfg["head_dim"]
    QD, KD, F, V, C = cfg["n_head"] * HD, cfg["n_kv_head"] * HD, cfg["d_ff"], cfg["vocab"], cfg["ctx"]
    g = torch.Generator(device="cuda")

    def qrand(rows, k, sd, std=0.02):
        g.manual_seed(sd)
        out = torch.empty((rows, H.row_bytes(qt, k)), dtype=torch.uint8, device="cuda")
        step = max(1, (1 << 25) // k)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            H.quantize(qt, torch.randn((r1 - r0, k), generator=g, device="cuda").mul_(std), out=out[r0:r1])
        return out

    def norm_w(n, sd):
        g.manual_seed(sd)
        return (1.0 + 0.1 * torch.randn(n, generator=g, device="cuda")).float()

    dev_layers, host_layers = [], []
    for l in range(cfg["n_layer"]):
        sd = seed + 100 * l
        qkv, wo, gu, down = qrand(QD + 2 * KD, D, sd), qrand(D, QD, sd + 1), qrand(2 * F, D, sd + 2), \
            qrand(D, F, sd + 3)
        g.manual_seed(sd + 4)
        kc = torch.randn((C, KD), generator=g, device="cuda").half()
        vc = torch.randn((C, KD), generator=g, device="cuda").half()
        an, fn = norm_w(D, sd + 5), norm_w(D, sd + 6)
        dev_layers.append(dict(wq=qkv[:QD], wk=qkv[QD:QD + KD], wv=qkv[QD + KD:], wo=wo, w_gate=gu[:F],
                               w_up=gu[F:], w_down=down, attn_norm=an, ffn_norm=fn, k_cache=kc, v_cache=vc))
        hq = qkv.cpu().numpy()
        hg = gu.cpu().numpy()
        host_layers.append(dict(wq=np.ascontiguousarray(hq[:QD]), wk=np.ascontiguousarray(hq[QD:QD + KD]),
                                wv=np.ascontiguousarray(hq[QD + KD:]), wo=wo.cpu().numpy(),
                                w_gate=np.ascontiguousarray(hg[:F]), w_up=np.ascontiguousarray(hg[F:]),
                                w_down=down.cpu().numpy(), attn_norm=an.cpu().numpy(), ffn_norm=fn.cpu().numpy(),
                                k_cache=kc.cpu().numpy().view(np.uint16).copy(),
                                v_cache=vc.cpu().numpy().view(np.uint16).copy()))
    w_out = qrand(V, D, seed + 7)
    emb = qrand(V, D, seed + 8, std=1.0)
    out_norm = norm_w(D, seed + 9)
    return dev_layers, host_layers, w_out, emb, out_norm


def check_caches(cfg, dev_layers, host_layers, pos):
    slot = pos % cfg["ctx"]
    for d, w in zip(dev_layers, host_layers):
        for n in ("k_cache", "v_cache"):
            got = d[n].cpu().numpy().view(np.uint16)
            want = w[n]
            other = np.arange(cfg["ctx"]) != slot
            assert np.array_equal(got[other], want[other]), n
            gf = got[slot].view(np.float16).astype(np.float32)
            wf = want[slot].view(np.float16).astype(np.float32)
            np.testing.assert_allclose(gf, wf, rtol=2e-3, atol=1e-3)


@pytest.mark.parametrize("n_layer", [2, 32])
def test_decode_step_7b_widths_match_oracle(n_layer):
    import torch
    import hesa_cuda as H
    cfg = dict(CFG_7B, n_layer=n_layer)
    qt = cfg["qtype"]
    dev_layers, host_layers, w_out, emb, out_norm = build(cfg, seed=77)
    m = H.Model(cfg["n_layer"], cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["head_dim"], cfg["d_ff"],
                cfg["vocab"], cfg["ctx"], cfg["rms_eps"], cfg["rope_base"], qt)
    table = torch.from_numpy(H.rope_table(cfg["ctx"], cfg["head_dim"], cfg["rope_base"])).cuda()
    ws = H.decode_workspace(m)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    tok = 31999
    tok_dev = torch.tensor([tok], dtype=torch.int32, device="cuda")
    pos_dev = torch.tensor([POS], dtype=torch.int32, device="cuda")
    x = H.embed(qt, emb, cfg["d_model"], tok_dev)
    H.decode_step(m, H.make_layers(dev_layers), out_norm, w_out, table, x, pos_dev, logits, ws)
    got = logits.cpu().numpy()

    x_ref = O.dequantize(qt, emb[tok:tok + 1].cpu().numpy(), cfg["d_model"])[0]
    assert np.array_equal(x.cpu().numpy(), x_ref)            # exact embedding row
    on, wo = out_norm.cpu().numpy(), w_out.cpu().numpy()
    # the exact result, measured with every sum in fp64, first (the fp32 run
    # after it leaves its own K/V rows in the host caches for check_caches)
    exact = O.decode_step(cfg, host_layers, on, wo, x_ref, POS, f64=True)
    want = O.decode_step(cfg, host_layers, on, wo, x_ref, POS)
    err, err_exact, ref_exact = rel_l2(got, want), rel_l2(got, exact), rel_l2(want, exact)
    if n_layer <= 8:
        assert err <= 1e-5, f"{n_layer} layers: logits rel L2 {err:.3e} against the oracle"
    else:
        # Through 32 layers the fp32 rounding of the reference's own step (a
        # sequential fp32 sum of 4096 or 11008 terms per output, ~3e-6 each)
        # compounds to ~1.6e-5 of the exact logits, more than the bar itself.
        # The bar is then held against the exact result, and the kernels must
        # be at least as close to it as the reference's arithmetic is.
        assert err_exact <= 1e-5, f"{n_layer} layers: rel L2 {err_exact:.3e} against the exact logits"
        assert err_exact <= ref_exact, f"kernels {err_exact:.3e} vs the reference's fp32 {ref_exact:.3e}"
        assert err <= 3e-5, f"{n_layer} layers: rel L2 {err:.3e} against the oracle"
    check_caches(cfg, dev_layers, host_layers, POS)
    assert H.device_status() == 0
