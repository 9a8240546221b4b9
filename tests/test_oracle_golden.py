"""Pin the CPU oracle against the reference's own known answers (CPU only).

Fixtures (tests/golden/, made by tests/golden/gen_golden.py):
  w8_quantizer.npz              outputs of the reference's W8 encoder
                                (benchmarks/quantize_qwen3_5_w8.py, executed)
  reference_known_answers.json  the reference's native F64 known-answer tests
Each test uses the tolerance the reference test uses.
"""
import json

import numpy as np
import pytest

import oracle


def _f(v):
    return np.array([float(x) for x in v], dtype=np.float64)


@pytest.fixture(scope="module")
def ka(golden_dir):
    with open(golden_dir / "reference_known_answers.json") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def w8(golden_dir):
    return np.load(golden_dir / "w8_quantizer.npz")


# ------------------------------------------------------------- W8 storage

@pytest.mark.parametrize("group", [128, 64, 32])
@pytest.mark.parametrize("tensor", ["a", "b"])
def test_quantizer_matches_reference_encoder(w8, tensor, group):
    w = w8[f"{tensor}_g{group}_w"]
    q, s = oracle.quantize_w8(w, group)
    np.testing.assert_array_equal(s, w8[f"{tensor}_g{group}_s"])
    np.testing.assert_array_equal(q, w8[f"{tensor}_g{group}_q"])


def test_quantizer_edge_rows(w8):
    q = w8["a_g128_q"]
    assert (q[3] == 128).all()                     # zero row: scale clamp, q = 0
    assert q[4, 0] == 1 and q[4, 1] == 128 and q[4, 2] == 130  # -127, tie->0, tie->2
    assert q.min() >= 1 and q.max() <= 255          # q in [-127, 127]


# --------------------------------------------------------- QuantizedLinear

def test_w8_linear_modes_on_reference_encoding(w8):
    """layers.rs:257-298 semantics on the reference encoder's own output."""
    w, q, s = w8["b_g32_w"], w8["b_g32_q"], w8["b_g32_s"]
    x = oracle.normal(3 * 128, 7).reshape(3, 128)
    deq = (q.astype(np.float32) - 128.0).reshape(5, 4, 32) * s[:, :, None]
    deq = deq.reshape(5, 128).astype(np.float32)
    ref_f32 = x.astype(np.float64) @ deq.astype(np.float64).T
    np.testing.assert_allclose(oracle.w8_linear(x, q, s, 32, mode=0), ref_f32, rtol=1e-6, atol=1e-6)
    xb = oracle.bf16_round(x).astype(np.float64)
    db = oracle.bf16_round(deq).astype(np.float64)
    ref_bf16 = oracle.bf16_round((xb @ db.T).astype(np.float32))
    np.testing.assert_array_equal(oracle.w8_linear(x, q, s, 32, mode=1), ref_bf16)
    # mode 2 = exact factored algebra; agrees with f32 mode up to bf16(x)
    exact = (xb @ deq.astype(np.float64).T)
    np.testing.assert_allclose(oracle.w8_linear(x, q, s, 32, mode=2), exact, rtol=1e-6, atol=1e-7)


def test_linear_known_answers(ka):
    case = ka["linear"]
    w = np.array(case["weight"], np.float32).reshape(2, 3)
    for c in case["cases"]:
        x = np.array(c["x"], np.float32).reshape(-1, 3)
        y = oracle.linear(x, w).reshape(-1)
        e = np.array(c["expected"])
        assert np.all(np.abs(y - e) <= case["rel_tolerance"] * np.maximum(np.abs(e), 1.0))


# -------------------------------------------------------------- attention

def test_gqa_known_answers(ka):
    case = ka["gqa"]
    for c in case["cases"]:
        kvh = c["kv_heads"]
        q = np.array(c["q"], np.float32).reshape(2, 4, 3, 2)
        k = np.array(c["k"], np.float32).reshape(2, kvh, 4, 2)
        v = np.array(c["v"], np.float32).reshape(2, kvh, 4, 3)
        mask = _f(c["mask"]).astype(np.float32).reshape(1, 4, 3, 4)
        out = oracle.gqa_attention(q, k, v, mask).reshape(-1)
        np.testing.assert_allclose(out, c["expected"], rtol=0, atol=case["tolerance"])


def test_masked_decode_known_answers(ka):
    """Stateful decode: cache starts at 100/1000, written at `position`, masked."""
    case = ka["masked_decode"]
    kc = np.full((2, 4, 2), case["cache_k_init"], np.float32)
    vc = np.full((2, 4, 2), case["cache_v_init"], np.float32)
    for st in case["steps"]:
        pos = st["position"]
        ku = np.array(st["k"], np.float32).reshape(2, 1, 2)
        vu = np.array(st["v"], np.float32).reshape(2, 1, 2)
        assert oracle.kv_update(kc, vc, ku, vu, [0, pos, 0]) == 1
        q = np.array(st["q"], np.float32).reshape(1, 2, 1, 2)
        mask = oracle.causal_mask([pos], np.arange(4))
        out = oracle.gqa_attention(q, kc.reshape(1, 2, 4, 2), vc.reshape(1, 2, 4, 2), mask)
        np.testing.assert_allclose(out.reshape(-1), st["expected_out"], atol=case["tolerance"])


def test_attention_broadcast_and_scales(ka):
    case = ka["attention"]["broadcast"]
    q = np.array(case["q"], np.float32).reshape(2, 1, 1, 2)
    k = np.array(case["k"], np.float32).reshape(1, 1, 3, 2)
    v = np.array(case["v"], np.float32).reshape(2, 1, 3, 1)
    mask = _f(case["mask"]).astype(np.float32)
    for scale, expected in zip(case["scales"], case["expected"]):
        for b in range(2):
            out = oracle.gqa_attention(q[b:b + 1], k, v[b:b + 1], mask, scale=scale)
            assert abs(out.reshape(-1)[0] - expected[b]) < 2e-6


def test_multihead_attention(ka):
    case = ka["attention"]["multihead"]
    q = np.array(case["q"], np.float32).reshape(2, 3, 4, 2)
    k = np.array(case["k"], np.float32).reshape(2, 3, 5, 2)
    v = np.array(case["v"], np.float32).reshape(2, 3, 5, 2)
    out = oracle.gqa_attention(q, k, v).reshape(-1)
    np.testing.assert_allclose(out, case["expected_y"], atol=2e-6)


def test_causal_mask_known_answers(ka):
    case = ka["causal"]
    ex = case["extreme_positions"]
    np.testing.assert_array_equal(oracle.causal_mask(ex["q"], ex["k"]).reshape(-1),
                                  _f(ex["expected"]).astype(np.float32))
    om = case["offset_mask"]
    qpos = np.arange(om["queries"]) + om["offset"]
    np.testing.assert_array_equal(oracle.causal_mask(qpos, np.arange(om["keys"])).reshape(-1),
                                  _f(om["expected"]).astype(np.float32))


def test_causal_runtime_positions(ka):
    case = ka["causal"]["runtime_positions"]
    v = np.array(case["values"], np.float32).reshape(1, 1, 4, 1)
    for c in case["cases"]:
        mask = oracle.causal_mask(c["q"], case["keys"])
        q = np.zeros((1, 1, 2, 1), np.float32)
        k = np.zeros((1, 1, 4, 1), np.float32)
        out = oracle.gqa_attention(q, k, v, mask, scale=1.0).reshape(-1)
        np.testing.assert_allclose(out, c["expected"], atol=ka["causal"]["tolerance"])


def test_full_and_chunked_causal(ka):
    case = ka["causal"]["full"]
    q = np.array(case["q"], np.float32).reshape(1, 1, 5, 2)
    k = np.array(case["k"], np.float32).reshape(1, 1, 7, 2)
    v = np.array(case["v"], np.float32).reshape(1, 1, 7, 2)
    full = oracle.gqa_attention(q, k, v, oracle.causal_mask(np.arange(5), np.arange(7)), scale=1.0)
    np.testing.assert_allclose(full.reshape(-1), case["expected"], atol=2e-5)
    for s, e in case["chunks"]:
        chunk = oracle.gqa_attention(q[:, :, s:e], k, v,
                                     oracle.causal_mask(np.arange(s, e), np.arange(7)), scale=1.0)
        np.testing.assert_allclose(chunk.reshape(-1), full[0, 0, s:e].reshape(-1), atol=2e-5)


# --------------------------------------------------------------- KV cache

def test_kv_cache_clamps_positions(ka):
    case = ka["kv_cache"]["clamp"]
    kc = np.zeros(case["cache_shape"], np.float32)
    vc = np.zeros(case["cache_shape"], np.float32)
    for pos, kv, vv in case["updates"]:
        assert oracle.kv_update(kc, vc, np.array([[kv]], np.float32), np.array([[vv]], np.float32),
                                [pos, 0]) == 1
    np.testing.assert_array_equal(kc.reshape(-1), case["expected_k"])
    np.testing.assert_array_equal(vc.reshape(-1), case["expected_v"])


def test_kv_cache_checked_keeps_pair(ka):
    case = ka["kv_cache"]["checked"]
    kc = np.zeros(case["cache_shape"], np.float32)
    vc = np.zeros(case["cache_shape"], np.float32)
    for st in case["steps"]:
        k = _f(st["k"]).astype(np.float32).reshape(2, 2)
        v = _f(st["v"]).astype(np.float32).reshape(2, 2)
        acc = oracle.kv_update(kc, vc, k, v, [st["row"], st["col"]], checked=True)
        assert acc == (1 if st["valid"] else 0)
        np.testing.assert_array_equal(kc.reshape(-1), st["expected_k"])
        np.testing.assert_array_equal(vc.reshape(-1), st["expected_v"])


# ------------------------------------------------------------------- RoPE

def test_rotary_tables(ka):
    case = ka["rotary"]
    x = np.array(case["values"], np.float32).reshape(6, 4)
    for t in case["tables"]:
        cos = np.array(t["cos"], np.float32).reshape(3, 2)
        sin = np.array(t["sin"], np.float32).reshape(3, 2)
        cos6 = np.concatenate([cos, cos])
        sin6 = np.concatenate([sin, sin])
        for layout in (0, 1):
            y = oracle.rope_cos_sin(x, cos6, sin6, layout).reshape(-1)
            np.testing.assert_allclose(y, t["expected"][str(layout)], atol=case["tolerance"])


def test_rotary_positions(ka):
    case = ka["rotary"]
    x = np.array(case["values_positions"], np.float32).reshape(2, 3, 4)
    for c in case["position_cases"]:
        pos = np.array(c["positions"], np.float32)
        fr = np.array(c["frequencies"], np.float32)
        ang = (pos[:, None] * fr[None, :]).astype(np.float32)
        cos = np.cos(ang.astype(np.float64)).astype(np.float32)
        sin = np.sin(ang.astype(np.float64)).astype(np.float32)
        for layout in (0, 1):
            y = oracle.rope_cos_sin(x.reshape(6, 4), np.concatenate([cos, cos]),
                                    np.concatenate([sin, sin]), layout).reshape(-1)
            np.testing.assert_allclose(y, c["expected"][str(layout)], atol=case["position_tolerance"])


def test_rope_split_half_positions_match_table_form():
    inv = oracle.rope_inv_freq(1e6, 64)
    assert inv[0] == 1.0 and inv.dtype == np.float32
    x = oracle.normal(3 * 64, 11).reshape(3, 64)
    pos = np.array([0, 5, 4097], np.int32)
    y = oracle.rope_split_half(x, pos, inv)
    ang = (pos.astype(np.float32)[:, None] * inv[None, :]).astype(np.float32)
    y2 = oracle.rope_cos_sin(x, np.cos(ang.astype(np.float64)).astype(np.float32),
                             np.sin(ang.astype(np.float64)).astype(np.float32), 0)
    np.testing.assert_array_equal(y, y2)
    np.testing.assert_array_equal(y[0], x[0])  # position 0 is the identity


# ---------------------------------------------------- paged decode contract

def _paged_case(batch=3, hq=8, hkv=2, d=64, ctx=(5, 16, 40), pages=12, seed=3):
    rng = np.random.default_rng(seed)
    max_pages = 4
    pt = rng.permutation(pages)[: batch * max_pages].reshape(batch, max_pages).astype(np.int32)
    kp = oracle.f32_to_bf16_bits(oracle.normal(pages * hkv * 16 * d, seed + 1).reshape(pages, hkv, 16, d))
    vp = oracle.f32_to_bf16_bits(oracle.normal(pages * hkv * 16 * d, seed + 2).reshape(pages, hkv, 16, d))
    q = oracle.bf16_round(oracle.normal(batch * hq * d, seed + 3).reshape(batch, hq * d))
    kn = oracle.bf16_round(oracle.normal(batch * hkv * d, seed + 4).reshape(batch, hkv * d))
    vn = oracle.bf16_round(oracle.normal(batch * hkv * d, seed + 5).reshape(batch, hkv * d))
    return dict(pt=pt, kp=kp, vp=vp, q=q, kn=kn, vn=vn, ctx=np.array(ctx, np.int32), hq=hq,
                hkv=hkv, d=d)


def test_paged_decode_matches_dense_gqa():
    c = _paged_case()
    kp, vp, ctx = c["kp"].copy(), c["vp"].copy(), c["ctx"].copy()
    inv = oracle.rope_inv_freq(1e6, c["d"])
    out, acc = oracle.paged_decode_attention(
        q=c["q"], k_new=c["kn"], v_new=c["vn"], k_pages=kp, v_pages=vp, page_table=c["pt"],
        ctx_lens=ctx, hq=c["hq"], hkv=c["hkv"], d=c["d"], inv_freq=inv, rotary_dim=c["d"],
        advance_ctx=True)
    assert (acc == 1).all() and (ctx == c["ctx"] + 1).all()
    d, hkv, hq = c["d"], c["hkv"], c["hq"]
    for b in range(3):
        pos = int(c["ctx"][b])
        n = pos + 1
        slots = np.arange(n)
        pages = c["pt"][b][slots // 16]
        K = oracle.bf16_bits_to_f32(kp[pages, :, slots % 16]).transpose(1, 0, 2)  # [hkv, n, d]
        V = oracle.bf16_bits_to_f32(vp[pages, :, slots % 16]).transpose(1, 0, 2)
        qr = oracle.rope_split_half(c["q"][b].reshape(hq, d), np.full(hq, pos), inv)
        kr = oracle.rope_split_half(c["kn"][b].reshape(hkv, d), np.full(hkv, pos), inv)
        np.testing.assert_array_equal(K[:, pos], oracle.bf16_round(kr))
        ref = oracle.gqa_attention(qr.reshape(1, hq, 1, d), K[None], V[None]).reshape(hq * d)
        np.testing.assert_allclose(out[b], oracle.bf16_round(ref), rtol=1e-2, atol=1e-6)


def test_paged_decode_checked_rejects_and_clamp_overwrites():
    c = _paged_case(ctx=(64, 63, 70))  # capacity 4 pages * 16 = 64
    for mode in (0, 1):
        kp, vp, ctx = c["kp"].copy(), c["vp"].copy(), c["ctx"].copy()
        out, acc = oracle.paged_decode_attention(
            q=c["q"], k_new=c["kn"], v_new=c["vn"], k_pages=kp, v_pages=vp, page_table=c["pt"],
            ctx_lens=ctx, hq=c["hq"], hkv=c["hkv"], d=c["d"], kv_update=mode, advance_ctx=True)
        if mode == 1:
            assert acc.tolist() == [0, 1, 0]
            assert ctx.tolist() == [64, 64, 70]
            # rejected sequences leave their pages untouched
            p = c["pt"][0][3]
            np.testing.assert_array_equal(kp[p], c["kp"][p])
        else:
            assert acc.tolist() == [1, 1, 1]
            p = c["pt"][0][3]
            np.testing.assert_array_equal(kp[p, :, 15], oracle.f32_to_bf16_bits(c["kn"][0].reshape(2, 64)))
        assert np.isfinite(out).all()


# ------------------------------------------------------------------ decoder

def test_tiny_decoder_runs_and_is_deterministic():
    cfg = dict(layers=1, hidden=64, q_heads=4, kv_heads=2, head_dim=16, intermediate=96,
               vocab=128, max_batch=2, max_context=16)
    outs = []
    for _ in range(2):
        dec = oracle.Decoder(**cfg)
        dec.init_synthetic(0)
        toks = np.array([3, 77], np.int32)
        seq = []
        for _ in range(4):
            logits, toks = dec.step(toks)
            seq.append(toks.copy())
        outs.append((np.stack(seq), logits))
        dec.close()
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    assert np.isfinite(outs[0][1]).all()


@pytest.mark.parametrize("emb_bf16,group", [(True, 0), (False, 128)])
def test_stepped_decoder_equals_full_sequence_causal_forward(emb_bf16, group):
    """The oracle decoder stepped one token at a time (what the GPU prefill and
    decode tests compare against) gives the same last-row logits and token as
    the full-sequence forward under the causal mask — the reference's prompt
    path (qwen3_5/mod.rs:199-260 with the mask of :229).  Both read K/V
    rounded to bf16 and sum in the same order, so they agree exactly."""
    cfg = dict(layers=2, hidden=512, q_heads=8, kv_heads=2, head_dim=64, intermediate=1536,
               vocab=4096)
    dec = oracle.Decoder(**cfg, embedding_bf16=emb_bf16, group_size=group, max_batch=1,
                         max_context=64)
    dec.init_synthetic(17)
    prompt = oracle.randint(24, 3, 0, cfg["vocab"])
    full_logits, full_tok = dec.forward(prompt)
    for t in prompt:
        step_logits, step_tok = dec.step(np.array([t], np.int32))
    np.testing.assert_array_equal(full_logits, step_logits[0])
    assert full_tok == int(step_tok[0])
    dec.close()


def test_oracle_prefill_equals_stepping_bit_for_bit():
    """Decoder.prefill (the full-sequence forward that also fills the cache)
    leaves the same state as stepping the prompt token by token: the last
    prompt row's logits and every later decode step are bit-identical."""
    import numpy as np
    cfg = dict(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=64, intermediate=512,
               vocab=1024)
    a = oracle.Decoder(**cfg, max_batch=1, max_context=64)
    b = oracle.Decoder(**cfg, max_batch=1, max_context=64)
    a.init_synthetic(2)
    b.init_synthetic(2)
    prompt = oracle.randint(24, 3, 0, 1024)
    for t in prompt:
        la, _ = a.step(np.array([t], np.int32))
    lb, _ = b.prefill(0, prompt)
    assert np.array_equal(la[0].view(np.uint32), lb.view(np.uint32))
    for t in (5, 17, 900):
        la, _ = a.step(np.array([t], np.int32))
        lb, _ = b.step(np.array([t], np.int32))
        assert np.array_equal(la.view(np.uint32), lb.view(np.uint32))
    a.close()
    b.close()
