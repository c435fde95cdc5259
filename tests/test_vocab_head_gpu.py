"""The vocabulary-parallel output head against the single-GPU head.

The head's rows are split over P "stages" (here P Stage objects on one GPU,
each holding only its rows); each computes dial_decoder_head_shard (final
norm, GEMV, greedy key per row) and dial_head_merge picks the token.  Checked
against dial_decoder_head on the full head (itself parity-tested against the
oracle in the model tests): the merged tokens equal its argmax, and every
shard's logits equal the full logits' slice bit for bit -- for the W8A16 head
(f16 and bf16 activations; the GEMV writes the keys in its epilogue), the
GGUF Q8_0 head of the Llama config (keys from the logits), ties across shards
(the first index wins, as argmax), rows selected by row_index (the prefill
form), and uneven shares including empty ones.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch(cuda):
    import torch as _t
    return _t


def _head_weights(torch, cfg, tie_rows, seed=7):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn((cfg.vocab, cfg.hidden), generator=g, device="cuda") * cfg.init_std
    pattern = torch.where(torch.arange(cfg.hidden, device="cuda") % 3 == 0, 0.08, -0.01)
    for r in tie_rows:  # identical rows: identical logits in different shards
        w[r] = pattern
    return w


def _check(torch, cfg, shares, rows=3, row_index=False, tie_rows=()):
    from dial_cuda.model import Stage, head_merge, vocab_shards
    L = cfg.n_layers
    w = _head_weights(torch, cfg, tie_rows)
    weights = {("lm_head",): w}
    full = Stage(cfg, L, L, n_slots=1, max_seq=16, with_embed=False, with_head=True, weights=weights)
    spans = vocab_shards(cfg.vocab, shares)
    shards = [Stage(cfg, L, L, n_slots=1, max_seq=16, with_embed=False, with_head=False,
                    weights=weights, head_rows=sp) for sp in spans]
    g = torch.Generator(device="cuda").manual_seed(11)
    T = rows + 2 if row_index else rows
    hidden = (torch.randn((T, cfg.hidden), generator=g, device="cuda") * 2).to(full.dt)
    if tie_rows:  # make the tied rows win: hidden aligned with their pattern
        hidden[:, ::3] = 3.0
    idx = torch.tensor([T - 1, 0, 2][:rows], dtype=torch.int32, device="cuda") if row_index else None
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    logits = torch.empty((rows, cfg.vocab), dtype=full.dt, device="cuda")
    full.head_forward(hidden, ids, row_index=idx, logits=logits)
    keys = torch.zeros((len(spans), rows), dtype=torch.int64, device="cuda")
    for k, (st, (v0, v1)) in enumerate(zip(shards, spans)):
        if v1 == v0:
            continue  # an empty share contributes key 0
        lg = torch.empty((rows, v1 - v0), dtype=full.dt, device="cuda")
        st.head_shard_forward(hidden, keys[k], row_index=idx, logits=lg)
        assert torch.equal(lg.view(torch.int16), logits[:, v0:v1].view(torch.int16)), (v0, v1)
    merged = torch.empty(rows, dtype=torch.int32, device="cuda")
    head_merge(keys, merged)
    torch.cuda.synchronize()
    want = ids.cpu().numpy()
    assert np.array_equal(merged.cpu().numpy(), want), (merged.cpu().numpy(), want)
    # the argmax of the returned logits, first index on ties
    lf = logits.float().cpu().numpy()
    assert np.array_equal(want, lf.argmax(axis=1))
    if tie_rows:
        assert (want == min(tie_rows)).all()
    import dial_cuda as D
    assert D.lib().dial_device_error(1) == 0


@pytest.mark.parametrize("act", ["f16", "bf16"])
@pytest.mark.parametrize("P", [2, 3, 8])
def test_w8a16_head_shards_merge_to_the_full_argmax(torch, act, P):
    from dial_cuda.model import ModelConfig
    _check(torch, ModelConfig(act_dtype=act), [1] * P)


def test_ties_across_shards_pick_the_first_index(torch):
    from dial_cuda.model import ModelConfig
    _check(torch, ModelConfig(), [1, 1, 1, 1], tie_rows=(100000, 5, 140000))


def test_uneven_and_empty_shares_and_row_index(torch):
    from dial_cuda.model import ModelConfig
    _check(torch, ModelConfig(), [0, 3, 1, 0, 2], row_index=True)


def test_q8_0_head_shards(torch):
    from dial_cuda.model import ModelConfig
    _check(torch, ModelConfig.llama3_8b_q4_0(), [1, 2, 1], rows=2)
