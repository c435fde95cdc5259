"""GPU parity of the decoder glue and of whole-model greedy decoding.

* glue ops through the C ABI against the oracle / numpy restatements:
  RMSNorm(+residual) (residual sum bit-exact, output within f16 rounding),
  RoPE tables, QK-norm+RoPE+KV append, GQA attention (decode and causal
  prefill, chunked and unchunked), SwiGLU, embedding, argmax;
* greedy decoding: a small Qwen3-shaped model (head_dim 128, GQA 4:1, QK-norm,
  W8A16 weights quantised on the GPU, bit-exact with the oracle's) against the
  oracle decoder -- the first 32 generated tokens must match exactly (north
  star), with the oracle's top1-top2 margins printed on failure;
* full Qwen3-8B shape (36 layers, vocab 151936): size-independent properties --
  determinism, and the prefill (tcgen05 GEMM) and decode (skinny) paths giving
  the same next token and logits within 1e-2.
"""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def D(cuda):
    import dial_cuda
    return dial_cuda


@pytest.fixture(scope="module")
def torch(cuda):
    import torch as _t
    return _t


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


# ---------------------------------------------------------------- glue ops
@pytest.mark.parametrize("rows,dim", [(1, 4096), (7, 1000), (64, 4096)])
def test_rmsnorm_residual(D, torch, rows, dim):
    rng = np.random.default_rng(rows + dim)
    x = rng.normal(0, 1, (rows, dim)).astype(np.float16)
    r = rng.normal(0, 3, (rows, dim)).astype(np.float16)
    w = (1 + 0.1 * rng.normal(0, 1, dim)).astype(np.float16)
    h_ref, y_ref = O.rmsnorm(x, w, 1e-6, res=r)
    xt, rt, wt = dev(torch, x), dev(torch, r), dev(torch, w)
    y = torch.empty_like(xt)
    D.check(D.lib().dial_rmsnorm(xt.data_ptr(), rt.data_ptr(), rt.data_ptr(), wt.data_ptr(),
                                 y.data_ptr(), D.F16, rows, dim, 1e-6, D.stream_ptr()), "rmsnorm")
    assert np.array_equal(rt.cpu().numpy().view(np.uint16), h_ref.view(np.uint16))  # in place, exact
    assert rel(y.cpu().numpy(), y_ref) <= 2e-3
    _, y0 = O.rmsnorm(x, w, 1e-6)
    y2 = torch.empty_like(xt)
    D.check(D.lib().dial_rmsnorm(xt.data_ptr(), None, None, wt.data_ptr(), y2.data_ptr(), D.F16, rows,
                                 dim, 1e-6, D.stream_ptr()), "rmsnorm")
    assert rel(y2.cpu().numpy(), y0) <= 2e-3


def test_rope_tables(D, torch):
    c_ref, s_ref = O.rope_tables(2048, 128, 1e6)
    c = torch.empty((2048, 64), dtype=torch.float16, device="cuda")
    s = torch.empty_like(c)
    D.check(D.lib().dial_rope_tables(c.data_ptr(), s.data_ptr(), D.F16, 2048, 128, 1e6, D.stream_ptr()),
            "rope")
    assert np.abs(c.cpu().numpy().astype(np.float32) - c_ref.astype(np.float32)).max() <= 1e-3
    assert np.abs(s.cpu().numpy().astype(np.float32) - s_ref.astype(np.float32)).max() <= 1e-3


def _rope_ref(v, cos_t, sin_t, p):
    """candle's rope over f16 tensors: every product and sum rounded to f16."""
    half = v.shape[-1] // 2
    c = cos_t[p].astype(np.float32)
    s = sin_t[p].astype(np.float32)
    a, b = np.asarray(v[..., :half], np.float32), np.asarray(v[..., half:], np.float32)
    r = lambda x: x.astype(np.float16).astype(np.float32)
    return np.concatenate([r(a * c) - r(b * s), r(a * s) + r(b * c)], -1).astype(np.float16)


@pytest.mark.parametrize("qk_norm", [1, 0])
def test_qk_norm_rope_kv_append(D, torch, qk_norm):
    rng = np.random.default_rng(11 + qk_norm)
    T, Hq, Hkv, Dh, S, slots = 5, 8, 2, 128, 64, 3
    qkv = rng.normal(0, 1, (T, (Hq + 2 * Hkv) * Dh)).astype(np.float16)
    qn = (1 + 0.1 * rng.normal(0, 1, Dh)).astype(np.float16)
    kn = (1 + 0.1 * rng.normal(0, 1, Dh)).astype(np.float16)
    pos = np.array([0, 1, 2, 17, 63], np.int32)
    slot = np.array([0, 0, 0, 2, 1], np.int32)
    cos_t, sin_t = O.rope_tables(S, Dh, 1e6)
    q_out = torch.empty((T, Hq, Dh), dtype=torch.float16, device="cuda")
    kc = torch.zeros((slots, Hkv, S, Dh), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    # device copies stay referenced until the kernel has run (a temporary's memory
    # would go back to the caching allocator as soon as data_ptr() returned)
    t_in = [dev(torch, a) for a in (qkv, qn, kn, cos_t, sin_t, pos, slot)]
    D.check(D.lib().dial_qk_norm_rope_kv_append(
        *[t.data_ptr() for t in t_in], q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), D.F16, T, Hq,
        Hkv, Dh, S, 1e-6, qk_norm, D.stream_ptr()), "qk_rope")
    torch.cuda.synchronize()
    qkv32 = qkv.astype(np.float32).reshape(T, Hq + 2 * Hkv, Dh)
    qo, kco, vco = q_out.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()
    for t in range(T):
        heads = qkv32[t].copy()
        if qk_norm:
            for h in range(Hq + Hkv):
                x = heads[h]
                w = qn if h < Hq else kn
                heads[h] = (x / np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-6) * w).astype(np.float16)
        rq = _rope_ref(heads[:Hq], cos_t, sin_t, pos[t])
        rk = _rope_ref(heads[Hq:Hq + Hkv], cos_t, sin_t, pos[t])
        if qk_norm:
            assert rel(qo[t], rq) <= 3e-3
            assert rel(kco[slot[t], :, pos[t]], rk) <= 3e-3
        else:  # RoPE alone: the same f16 operations, bit-exact
            assert np.array_equal(qo[t].view(np.uint16), rq.view(np.uint16))
            assert np.array_equal(kco[slot[t], :, pos[t]].view(np.uint16), rk.view(np.uint16))
        assert np.array_equal(vco[slot[t], :, pos[t]], qkv[t].reshape(-1, Dh)[Hq + Hkv:])


def _round_dt(x, dt):
    """Round to the activation type (float64 values out)."""
    x = np.asarray(x, np.float32)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float64)
    if dt == "bf16":
        return O.bf16_to_f32(O.f32_to_bf16(x)).astype(np.float64)
    return x.astype(np.float64)


def _attn_ref(q, kc, vc, pos, slot, Hkv, dt):
    """The reference's attention (text.rs:1278-1280): s = T(T(q.k) * T(1/sqrt(D))),
    softmax, o = p.V (probabilities unrounded, see the kernel's note)."""
    T, Hq, Dh = q.shape
    rep = Hq // Hkv
    mul = _round_dt(1.0 / np.sqrt(Dh), dt)
    out = np.zeros((T, Hq, Dh))
    for t in range(T):
        for h in range(Hq):
            K = kc[slot[t], h // rep, :pos[t] + 1].astype(np.float64)
            V = vc[slot[t], h // rep, :pos[t] + 1].astype(np.float64)
            s = _round_dt(_round_dt(K @ q[t, h].astype(np.float64), dt) * mul, dt)
            p = np.exp(s - s.max())
            out[t, h] = p @ V / p.sum()
    return out.reshape(T, Hq * Dh)


def _cast(x, dt):
    """float32 array -> (array the kernel reads, float64 values it holds)."""
    if dt == "f16":
        h = x.astype(np.float16)
        return h, h.astype(np.float64)
    if dt == "bf16":
        b = O.f32_to_bf16(x)
        return b.view(np.int16), O.bf16_to_f32(b).astype(np.float64)
    return x.astype(np.float32), x.astype(np.float64)


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("mode,Hq", [("decode", 32), ("prefill", 32), ("long", 32), ("decode", 8),
                                     ("decode", 16), ("decode", 64), ("batched", 32)])
def test_attention(D, torch, mode, Hq, dt):
    """Decode (one token per sequence), prefill (causal run of one sequence),
    long contexts (several key splits + combine), n_rep 1/2/4/8, and the batched
    decode of 32 sequences with ~2k-token caches; f16/bf16 caches run on the
    tensor-core kernel."""
    rng = np.random.default_rng({"decode": 1, "prefill": 2, "long": 3, "batched": 4}[mode] + Hq)
    Hkv, Dh, slots = 8, 128, 4
    S = {"long": 1300, "batched": 2100}.get(mode, 256)
    if mode == "decode":
        pos = np.array([0, 5, 200, 255], np.int32)
        slot = np.array([0, 1, 2, 3], np.int32)
    elif mode == "prefill":
        pos = np.arange(40, dtype=np.int32)
        slot = np.full(40, 2, np.int32)
    elif mode == "long":  # several key splits, combine step
        pos = np.array([1299, 700, 511, 512], np.int32)
        slot = np.array([0, 1, 2, 3], np.int32)
    else:
        slots = 32
        pos = rng.integers(2000, 2100, 32).astype(np.int32)
        slot = rng.permutation(32).astype(np.int32)
    T = len(pos)
    q, q64 = _cast(rng.normal(0, 1, (T, Hq, Dh)).astype(np.float32), dt)
    kc, k64 = _cast(rng.normal(0, 1, (slots, Hkv, S, Dh)).astype(np.float32), dt)
    vc, v64 = _cast(rng.normal(0, 1, (slots, Hkv, S, Dh)).astype(np.float32), dt)
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    out = torch.empty((T, Hq * Dh), dtype=tdt, device="cuda")
    max_len = int(pos.max()) + 1
    need = D.lib().dial_attention_workspace_bytes(T, Hq, max_len)
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    t_in = [dev(torch, a) for a in (q, kc, vc, pos, slot)]
    code = {"f16": D.F16, "bf16": D.BF16, "f32": D.F32}[dt]
    outs = []
    for _ in range(2):  # repeated calls give bit-identical outputs
        D.check(D.lib().dial_attention(*[t.data_ptr() for t in t_in], out.data_ptr(),
                                       ws.data_ptr() if need else None, need, code, T, Hq, Hkv, Dh,
                                       S, max_len, D.stream_ptr()), "attention")
        outs.append(out.float().cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    ref = _attn_ref(q64, k64, v64, pos, slot, Hkv, dt)
    got = outs[0]
    # output rounding of the type (f16 2^-11, bf16 2^-8) plus f32 accumulation
    assert rel(got, ref) <= {"f16": 3e-3, "bf16": 1e-2}[dt]


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("Hq,Hkv,qk_norm", [(32, 8, 1), (32, 8, 0), (8, 8, 1), (16, 8, 1), (64, 8, 1),
                                            (16, 2, 1)])
def test_decode_attention_fused_matches_two_call_form(D, torch, dt, Hq, Hkv, qk_norm):
    """dial_decode_attention (one launch: QK-norm, RoPE, cache append, the key
    splits and their merge by the last split to finish) against
    dial_qk_norm_rope_kv_append + dial_attention on the same inputs: output and
    both caches bit-identical, for contexts from one key to many splits; one
    zero-filled workspace serves every call (its counters return to zero)."""
    rng = np.random.default_rng(Hq + Hkv + qk_norm + (dt == "bf16"))
    Dh, S, slots = 128, 4200, 3
    cos_t, sin_t = O.rope_tables(S, Dh, 1e6)
    if dt == "bf16":
        cos_t, sin_t = (O.f32_to_bf16(x.astype(np.float32)).view(np.int16) for x in (cos_t, sin_t))
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    code = {"f16": D.F16, "bf16": D.BF16}[dt]
    kc0, _ = _cast(rng.normal(0, 1, (slots, Hkv, S, Dh)).astype(np.float32), dt)
    vc0, _ = _cast(rng.normal(0, 1, (slots, Hkv, S, Dh)).astype(np.float32), dt)
    qn, _ = _cast((1 + 0.1 * rng.normal(0, 1, Dh)).astype(np.float32), dt)
    kn, _ = _cast((1 + 0.1 * rng.normal(0, 1, Dh)).astype(np.float32), dt)
    tabs = [dev(torch, a) for a in (qn, kn, cos_t, sin_t)]
    wsb = D.lib().dial_decode_attention_workspace_bytes(Hq, S)
    dws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    for p, sl in [(0, 1), (5, 0), (130, 2), (700, 1), (1299, 2), (4100, 0)]:
        qkv, _ = _cast(rng.normal(0, 1, (1, (Hq + 2 * Hkv) * Dh)).astype(np.float32), dt)
        qkv_t, pos_t, slot_t = dev(torch, qkv), dev(torch, np.array([p], np.int32)), \
            dev(torch, np.array([sl], np.int32))
        max_len = p + 1
        # two-call form
        kc_a, vc_a = dev(torch, kc0), dev(torch, vc0)
        q = torch.empty((1, Hq, Dh), dtype=tdt, device="cuda")
        out_a = torch.empty((1, Hq * Dh), dtype=tdt, device="cuda")
        D.check(D.lib().dial_qk_norm_rope_kv_append(
            qkv_t.data_ptr(), *[t.data_ptr() for t in tabs], pos_t.data_ptr(), slot_t.data_ptr(),
            q.data_ptr(), kc_a.data_ptr(), vc_a.data_ptr(), code, 1, Hq, Hkv, Dh, S, 1e-6, qk_norm,
            D.stream_ptr()), "qk_rope")
        need = D.lib().dial_attention_workspace_bytes(1, Hq, max_len)
        ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
        D.check(D.lib().dial_attention(q.data_ptr(), kc_a.data_ptr(), vc_a.data_ptr(), pos_t.data_ptr(),
                                       slot_t.data_ptr(), out_a.data_ptr(), ws.data_ptr() if need else None,
                                       need, code, 1, Hq, Hkv, Dh, S, max_len, D.stream_ptr()), "attention")
        # one launch
        kc_b, vc_b = dev(torch, kc0), dev(torch, vc0)
        out_b = torch.empty_like(out_a)
        for _ in range(2):  # the second call finds the counters back at zero
            D.check(D.lib().dial_decode_attention(
                qkv_t.data_ptr(), *[t.data_ptr() for t in tabs], pos_t.data_ptr(), slot_t.data_ptr(),
                kc_b.data_ptr(), vc_b.data_ptr(), out_b.data_ptr(), dws.data_ptr(), wsb, code, Hq, Hkv,
                Dh, S, max_len, 1e-6, qk_norm, D.stream_ptr()), "decode_attention")
            torch.cuda.synchronize()
            assert torch.equal(kc_a.view(torch.int16), kc_b.view(torch.int16)), p
            assert torch.equal(vc_a.view(torch.int16), vc_b.view(torch.int16)), p
            assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16)), p
    assert int(dws[wsb - 4 * Hq:].count_nonzero()) == 0
    assert D.lib().dial_device_error(1) == 0


def test_swiglu_embedding_argmax(D, torch):
    rng = np.random.default_rng(5)
    T, I = 3, 1000
    gu = rng.normal(0, 2, (T, 2 * I)).astype(np.float16)
    out = torch.empty((T, I), dtype=torch.float16, device="cuda")
    gut = dev(torch, gu)
    D.check(D.lib().dial_swiglu(gut.data_ptr(), out.data_ptr(), D.F16, T, I, D.stream_ptr()), "swiglu")
    g, u = gu[:, :I].astype(np.float32), gu[:, I:].astype(np.float32)
    s = (g / (1 + np.exp(-g))).astype(np.float16).astype(np.float32)
    assert rel(out.cpu().numpy(), (s * u).astype(np.float16)) <= 2e-3
    table = rng.normal(0, 1, (50, 64)).astype(np.float16)
    ids = np.array([3, 49, 0, 7], np.int32)
    emb = torch.empty((4, 64), dtype=torch.float16, device="cuda")
    tt, it = dev(torch, table), dev(torch, ids)
    D.check(D.lib().dial_embedding(tt.data_ptr(), it.data_ptr(), emb.data_ptr(), D.F16, 4, 50, 64,
                                   D.stream_ptr()), "embedding")
    assert np.array_equal(emb.cpu().numpy(), table[ids])
    assert D.lib().dial_device_error(1) == 0
    logits = rng.normal(0, 1, (3, 151936)).astype(np.float16)
    logits[1, 77] = logits[1, 5000] = 9.0  # tie -> first index
    am = torch.empty(3, dtype=torch.int32, device="cuda")
    lt = dev(torch, logits)
    D.check(D.lib().dial_argmax(lt.data_ptr(), am.data_ptr(), D.F16, 3, 151936, D.stream_ptr()),
            "argmax")
    assert list(am.cpu().numpy()) == [int(np.argmax(logits[i])) for i in range(3)]
    assert am.cpu().numpy()[1] == 77


def test_embedding_out_of_range_sets_flag(D, torch):
    table = torch.zeros((10, 16), dtype=torch.float16, device="cuda")
    ids = torch.tensor([3, 10], dtype=torch.int32, device="cuda")
    out = torch.ones((2, 16), dtype=torch.float16, device="cuda")
    D.check(D.lib().dial_embedding(table.data_ptr(), ids.data_ptr(), out.data_ptr(), D.F16, 2, 10, 16,
                                   D.stream_ptr()), "embedding")
    assert D.lib().dial_device_error(1) == 1  # DIAL_ERR_INVALID_ARG, then cleared
    assert D.lib().dial_device_error(1) == 0
    assert (out.cpu().numpy()[1] == 0).all()


# ---------------------------------------------------------------- whole decoder
MINI = dict(n_layers=2, hidden=1024, inter=2048, n_heads=8, n_kv=2, head_dim=128, vocab=4096,
            qk_norm=True, eps=1e-6, theta=1e6)


def _mini_weights(seed=7):
    rng = np.random.default_rng(seed)
    c = MINI
    H, I, Dh = c["hidden"], c["inter"], c["head_dim"]
    QKV = (c["n_heads"] + 2 * c["n_kv"]) * Dh
    w = {}
    for li in range(c["n_layers"]):
        w[(li, "qkv")] = rng.normal(0, 0.02, (QKV, H)).astype(np.float32)
        w[(li, "o")] = rng.normal(0, 0.02, (H, c["n_heads"] * Dh)).astype(np.float32)
        w[(li, "gate_up")] = rng.normal(0, 0.02, (2 * I, H)).astype(np.float32)
        w[(li, "down")] = rng.normal(0, 0.02, (H, I)).astype(np.float32)
        for n, dim in (("input_norm", H), ("post_norm", H), ("q_norm", Dh), ("k_norm", Dh)):
            w[(li, n)] = (1 + 0.1 * rng.normal(0, 1, dim)).astype(np.float16)
    w[("embed",)] = rng.normal(0, 1.0, (c["vocab"], H)).astype(np.float32)
    w[("final_norm",)] = (1 + 0.1 * rng.normal(0, 1, H)).astype(np.float16)
    w[("lm_head",)] = rng.normal(0, 0.02, (c["vocab"], H)).astype(np.float32)
    return w


def test_decoder_greedy_32_tokens_match_oracle(D, torch):
    from dial_cuda.model import Decoder, ModelConfig
    w = _mini_weights()
    c = MINI
    cfg = ModelConfig(n_layers=c["n_layers"], hidden=c["hidden"], intermediate=c["inter"],
                      n_heads=c["n_heads"], n_kv_heads=c["n_kv"], vocab=c["vocab"],
                      rope_theta=c["theta"])
    dec = Decoder(cfg, n_slots=2, max_seq=64,
                  weights={k: torch.from_numpy(np.asarray(v, np.float32)) if v.dtype == np.float32
                           else torch.from_numpy(v) for k, v in w.items()})
    rng = np.random.default_rng(99)
    prompt = rng.integers(0, c["vocab"], 16).astype(np.int32)
    n_new = 32
    # oracle: same int8 weights (quantiser bit-exact with the GPU's)
    layers = []
    for li in range(c["n_layers"]):
        L = {}
        for name, key in (("qkv", "qkv"), ("o", "o"), ("gate_up", "gu"), ("down", "down")):
            q, s, _ = O.w8a16_quantize(w[(li, name)])
            L[f"{key}_q"], L[f"{key}_s"] = q, s
        for n in ("input_norm", "post_norm", "q_norm", "k_norm"):
            L[n] = w[(li, n)]
        layers.append(L)
    hq, hs, _ = O.w8a16_quantize(w[("lm_head",)])
    want, margins = O.decoder_generate(c, layers, w[("embed",)].astype(np.float16), w[("final_norm",)],
                                       hq, hs, prompt, n_new)
    # GPU: prefill then one decode step per token, slot 1
    got = [int(dec.prefill(dev(torch, prompt), slot=1).item())]
    ids = torch.tensor(got, dtype=torch.int32, device="cuda")
    slots = torch.tensor([1], dtype=torch.int32, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    for step in range(1, n_new):
        pos = torch.tensor([len(prompt) + step - 1], dtype=torch.int32, device="cuda")
        dec.decode_step(ids, pos, slots, max_len=len(prompt) + step, out_ids=out)
        got.append(int(out.item()))
        ids.copy_(out)
    assert D.lib().dial_device_error(1) == 0
    assert got == list(want), (f"first mismatch at {next(i for i in range(n_new) if got[i] != want[i])};"
                               f" oracle margins {np.round(margins, 4).tolist()}")


@pytest.fixture(scope="module")
def full_model(D, torch):
    from dial_cuda.model import Decoder, ModelConfig
    return Decoder(ModelConfig(), n_slots=3, max_seq=256)


def test_full_size_prefill_and_decode_agree(D, torch, full_model):
    """Qwen3-8B shape: next token after a 64-token prompt via the prefill path
    (tcgen05 GEMM on all 64 rows) and via prefill(63) + one decode step
    (skinny kernels) -- same token, logits within 1e-2."""
    dec = full_model
    st = dec.stage
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, dec.cfg.vocab, 64).astype(np.int32)
    a = int(dec.prefill(dev(torch, prompt), slot=0).item())
    # logits of the last prompt position through the prefill path
    T = 64
    hidden = torch.empty((T, dec.cfg.hidden), device="cuda", dtype=st.dt)
    st.embed_tokens(dev(torch, prompt), hidden)
    st.layers_forward(hidden, torch.arange(T, dtype=torch.int32, device="cuda"),
                      torch.zeros(T, dtype=torch.int32, device="cuda"), T)
    la = torch.empty((1, dec.cfg.vocab), device="cuda", dtype=st.dt)
    oa = torch.empty(1, dtype=torch.int32, device="cuda")
    st.head_forward(hidden, oa, row_index=torch.tensor([T - 1], dtype=torch.int32, device="cuda"),
                    logits=la)
    # decode path on slot 1
    dec.prefill(dev(torch, prompt[:63]), slot=1)
    h1 = torch.empty((1, dec.cfg.hidden), device="cuda", dtype=st.dt)
    st.embed_tokens(dev(torch, prompt[63:]), h1)
    st.layers_forward(h1, torch.tensor([63], dtype=torch.int32, device="cuda"),
                      torch.tensor([1], dtype=torch.int32, device="cuda"), 64)
    lb = torch.empty((1, dec.cfg.vocab), device="cuda", dtype=st.dt)
    ob = torch.empty(1, dtype=torch.int32, device="cuda")
    st.head_forward(h1, ob, logits=lb)
    assert D.lib().dial_device_error(1) == 0
    la_np, lb_np = la.float().cpu().numpy(), lb.float().cpu().numpy()
    assert np.isfinite(la_np).all() and np.isfinite(lb_np).all()
    assert rel(lb_np, la_np) <= 1e-2
    top2 = np.sort(la_np[0])[-2:]
    if top2[1] - top2[0] > 2e-2 * np.abs(la_np).max():  # not a near-tie
        assert a == int(oa.item()) == int(ob.item())


def test_full_size_decode_is_deterministic(D, torch, full_model):
    dec = full_model
    prompt = np.random.default_rng(4).integers(0, dec.cfg.vocab, 32).astype(np.int32)
    runs = []
    for _ in range(2):
        toks = [int(dec.prefill(dev(torch, prompt), slot=2).item())]
        ids = torch.tensor(toks, dtype=torch.int32, device="cuda")
        out = torch.empty(1, dtype=torch.int32, device="cuda")
        for step in range(1, 8):
            dec.decode_step(ids, torch.tensor([31 + step], dtype=torch.int32, device="cuda"),
                            torch.tensor([2], dtype=torch.int32, device="cuda"), 32 + step, out)
            toks.append(int(out.item()))
            ids.copy_(out)
        runs.append(toks)
    assert runs[0] == runs[1]
