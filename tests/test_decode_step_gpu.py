"""Decode step (hesa_cuda_decode_step) against the oracle's decode step on a
small seeded Llama-shaped model: logits within rel-L2 1e-5, the KV slot the
step writes within one fp16 rounding, every other slot untouched. Covers the
joined (one matvec for Q|K|V and gate|up) and separate weight layouts,
consecutive tokens, the ring wrap past ctx, the embedding lookup and a CUDA
graph replayed at new positions."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=2, d_model=256, n_head=4, n_kv_head=2, head_dim=64, d_ff=512, vocab=384, ctx=64,
           rms_eps=1e-6, rope_base=10000.0)
ROPE_ROWS = 160


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def build_model(qt, seed=7, prefill=40, cfg=None):
    c = dict(cfg or CFG, qtype=qt)
    D, QD, KD, F, V = c["d_model"], c["n_head"] * c["head_dim"], c["n_kv_head"] * c["head_dim"], c["d_ff"], c["vocab"]
    layers = []
    for l in range(c["n_layer"]):
        s = seed * 100 + l * 10
        w = {n: O.quantize(qt, O.gaussian(shape, 0.02, s + i)) for i, (n, shape) in enumerate(
            [("wq", (QD, D)), ("wk", (KD, D)), ("wv", (KD, D)), ("wo", (D, QD)), ("w_gate", (F, D)),
             ("w_up", (F, D)), ("w_down", (D, F))])}
        w["attn_norm"] = (1.0 + 0.1 * O.gaussian((D,), 1.0, s + 7)).astype(np.float32)
        w["ffn_norm"] = (1.0 + 0.1 * O.gaussian((D,), 1.0, s + 8)).astype(np.float32)
        kc = np.zeros((c["ctx"], KD), np.uint16)
        vc = np.zeros((c["ctx"], KD), np.uint16)
        kc[:prefill] = O.fp32_to_fp16_bits(O.gaussian((prefill, KD), 1.0, s + 9))
        vc[:prefill] = O.fp32_to_fp16_bits(O.gaussian((prefill, KD), 1.0, s + 10))
        w["k_cache"], w["v_cache"] = kc, vc
        layers.append(w)
    out_norm = (1.0 + 0.1 * O.gaussian((D,), 1.0, seed + 1)).astype(np.float32)
    w_out = O.quantize(qt, O.gaussian((V, D), 0.02, seed + 2))
    emb = O.quantize(qt, O.gaussian((V, D), 1.0, seed + 3))
    return c, layers, out_norm, w_out, emb


def to_device(c, layers, out_norm, w_out, joined, rope_rows=ROPE_ROWS):
    import torch
    import hesa_cuda as H
    dev = "cuda"
    keep, per = [], []
    for w in layers:
        d = {}
        if joined:
            qkv = torch.from_numpy(np.concatenate([w["wq"], w["wk"], w["wv"]])).to(dev)
            gu = torch.from_numpy(np.concatenate([w["w_gate"], w["w_up"]])).to(dev)
            nq, nk = w["wq"].shape[0], w["wk"].shape[0]
            d["wq"], d["wk"], d["wv"] = qkv[:nq], qkv[nq:nq + nk], qkv[nq + nk:]
            nf = w["w_gate"].shape[0]
            d["w_gate"], d["w_up"] = gu[:nf], gu[nf:]
            keep += [qkv, gu]
        else:
            for n in ("wq", "wk", "wv", "w_gate", "w_up"):
                d[n] = torch.from_numpy(w[n]).to(dev)
        for n in ("wo", "w_down", "attn_norm", "ffn_norm"):
            d[n] = torch.from_numpy(w[n]).to(dev)
        for n in ("k_cache", "v_cache"):
            d[n] = torch.from_numpy(w[n].view(np.int16)).to(dev)
        per.append(d)
    m = H.Model(c["n_layer"], c["d_model"], c["n_head"], c["n_kv_head"], c["head_dim"], c["d_ff"], c["vocab"],
                c["ctx"], c["rms_eps"], c["rope_base"], c["qtype"])
    table = torch.from_numpy(H.rope_table(rope_rows, c["head_dim"], c["rope_base"])).to(dev)
    return dict(model=m, per=per, keep=keep, layers=H.make_layers(per), out_norm=torch.from_numpy(out_norm).to(dev),
                w_out=torch.from_numpy(w_out).to(dev), table=table, ws=H.decode_workspace(m),
                logits=torch.empty(c["vocab"], dtype=torch.float32, device=dev))


def gpu_step(g, x, pos_dev):
    import hesa_cuda as H
    H.decode_step(g["model"], g["layers"], g["out_norm"], g["w_out"], g["table"], x, pos_dev, g["logits"], g["ws"])
    return g["logits"].cpu().numpy()


def check_caches(c, g, layers, pos):
    import torch
    slot = pos % c["ctx"]
    for d, w in zip(g["per"], layers):
        for n in ("k_cache", "v_cache"):
            got = d[n].cpu().numpy().view(np.uint16)
            want = w[n]
            other = np.arange(c["ctx"]) != slot
            assert np.array_equal(got[other], want[other]), n
            gf = got[slot].view(np.float16).astype(np.float32)
            wf = want[slot].view(np.float16).astype(np.float32)
            np.testing.assert_allclose(gf, wf, rtol=2e-3, atol=1e-3)


@pytest.mark.parametrize("qt,joined", [(O.Q4_K, True), (O.Q4_K, False), (O.Q8_0, True), (O.Q6_K, True)])
def test_decode_step_matches_oracle(qt, joined):
    import torch
    import hesa_cuda as H
    c, layers, out_norm, w_out, emb = build_model(qt, prefill=40)
    g = to_device(c, layers, out_norm, w_out, joined)
    emb_d = torch.from_numpy(emb).cuda()
    for step, (pos, tok) in enumerate([(40, 5), (41, 77), (42, 383)]):
        pos_dev = torch.tensor([pos], dtype=torch.int32, device="cuda")
        tok_dev = torch.tensor([tok], dtype=torch.int32, device="cuda")
        x = H.embed(qt, emb_d, c["d_model"], tok_dev)
        x_ref = O.dequantize(qt, emb[tok:tok + 1], c["d_model"])[0]
        assert np.array_equal(x.cpu().numpy(), x_ref)          # exact embedding row
        got = gpu_step(g, x, pos_dev)
        want = O.decode_step(c, layers, out_norm, w_out, x_ref, pos)
        err = rel_l2(got, want)
        assert err <= 1e-5, f"step {step} pos {pos}: rel L2 {err:.3e}"
        check_caches(c, g, layers, pos)
        # continue from the oracle's caches so both sides carry identical state
        for d, w in zip(g["per"], layers):
            for n in ("k_cache", "v_cache"):
                d[n].copy_(torch.from_numpy(w[n].view(np.int16)))
    assert H.device_status() == 0


# head_dim 128 (the 7B shape's) with four query heads per KV head and a context
# of four 128-slot splits; the last position wraps the ring
CFG_HD128 = dict(n_layer=2, d_model=512, n_head=8, n_kv_head=2, head_dim=128, d_ff=1024, vocab=512, ctx=512,
                 rms_eps=1e-6, rope_base=10000.0)


def test_decode_step_head_dim_128_gqa_matches_oracle():
    import torch
    import hesa_cuda as H
    qt = O.Q4_K
    c, layers, out_norm, w_out, emb = build_model(qt, seed=11, prefill=512, cfg=CFG_HD128)
    g = to_device(c, layers, out_norm, w_out, True, rope_rows=1024)
    emb_d = torch.from_numpy(emb).cuda()
    for step, (pos, tok) in enumerate([(300, 9), (511, 100), (700, 511)]):
        pos_dev = torch.tensor([pos], dtype=torch.int32, device="cuda")
        tok_dev = torch.tensor([tok], dtype=torch.int32, device="cuda")
        x = H.embed(qt, emb_d, c["d_model"], tok_dev)
        x_ref = O.dequantize(qt, emb[tok:tok + 1], c["d_model"])[0]
        got = gpu_step(g, x, pos_dev)
        want = O.decode_step(c, layers, out_norm, w_out, x_ref, pos)
        err = rel_l2(got, want)
        assert err <= 1e-5, f"step {step} pos {pos}: rel L2 {err:.3e}"
        check_caches(c, g, layers, pos)
        for d, w in zip(g["per"], layers):
            for n in ("k_cache", "v_cache"):
                d[n].copy_(torch.from_numpy(w[n].view(np.int16)))
    assert H.device_status() == 0


def test_decode_step_ring_wraps_and_graph_replays():
    import torch
    import hesa_cuda as H
    qt = O.Q4_K
    c, layers, out_norm, w_out, emb = build_model(qt, seed=11, prefill=64)
    g = to_device(c, layers, out_norm, w_out, True)
    x = torch.from_numpy(O.gaussian((c["d_model"],), 1.0, 99)).cuda()
    pos_dev = torch.tensor([0], dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        pos_dev.fill_(63)
        gpu_step(g, x, pos_dev)               # warm-up (eager), writes slot 63
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            H.decode_step(g["model"], g["layers"], g["out_norm"], g["w_out"], g["table"], x, pos_dev,
                          g["logits"], g["ws"], stream=stream)
    stream.synchronize()
    # reset both sides to the same caches, then replay at positions past ctx
    for d, w in zip(g["per"], layers):
        for n in ("k_cache", "v_cache"):
            d[n].copy_(torch.from_numpy(w[n].view(np.int16)))
    xr = x.cpu().numpy()
    for pos in (64, 65, 130):                 # slots 0, 1, 2 of the ring
        pos_dev.fill_(pos)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        got = g["logits"].cpu().numpy()
        want = O.decode_step(c, layers, out_norm, w_out, xr, pos)
        assert rel_l2(got, want) <= 1e-5, pos
        check_caches(c, g, layers, pos)
        for d, w in zip(g["per"], layers):
            for n in ("k_cache", "v_cache"):
                d[n].copy_(torch.from_numpy(w[n].view(np.int16)))
    del graph
    assert H.device_status() == 0


def test_decode_step_rejects_bad_arguments():
    import hesa_cuda as H
    c, layers, out_norm, w_out, emb = build_model(O.Q4_K, prefill=1)
    g = to_device(c, layers, out_norm, w_out, True)
    import torch
    pos_dev = torch.tensor([0], dtype=torch.int32, device="cuda")
    x = torch.zeros(c["d_model"], dtype=torch.float32, device="cuda")
    small = g["ws"][:64]
    with pytest.raises(H.HesaError) as ei:
        H.decode_step(g["model"], g["layers"], g["out_norm"], g["w_out"], g["table"], x, pos_dev, g["logits"], small)
    assert ei.value.code == 2
    bad = H.Model(0, 256, 4, 2, 64, 512, 384, 64, 1e-6, 1e4, O.Q4_K)
    assert H.lib().hesa_cuda_decode_workspace_size(bad) == 0
