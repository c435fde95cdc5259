"""Pipelined decode on the GPU.

- One stage (world 1): the pipeline's schedule and CUDA graphs give the same
  greedy tokens as Decoder.prefill/decode_step.
- Two stages over NCCL (needs 2 GPUs; skipped otherwise): each rank holds half
  the layers, the hand-off runs through the C ABI's stage communicators
  (dial_stage_comm_*), and the tokens equal the single-GPU ones (the weights of
  a layer do not depend on the split, and the arithmetic of a layer is the
  same).  Also with the vocabulary-parallel head: each rank holds half of the
  head's rows (both halves above the whole-tile GEMV's size, so each row's
  logit is computed exactly as on one GPU) and stage 0 merges the keys.
"""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SMALL = dict(n_layers=4, hidden=1024, intermediate=2048, n_heads=8, n_kv_heads=2, head_dim=128,
             vocab=4096, act_dtype="bf16")
N_MB, PROMPT, STEPS = 4, 24, 6


def _cfg(gguf: bool = False, vocab: int = SMALL["vocab"]):
    from dial_cuda.model import WFMT_Q4_0, WFMT_Q8_0, ModelConfig
    if gguf:  # the Llama-style GGUF decoder: Q4_0 layers, Q8_0 head, f16, no QK-norm
        return ModelConfig(**dict(SMALL, act_dtype="f16", qk_norm=False, rope_theta=5e5,
                                  weight_format=WFMT_Q4_0, head_format=WFMT_Q8_0, vocab=vocab))
    return ModelConfig(**dict(SMALL, vocab=vocab))


def _prompts(torch):
    rng = np.random.default_rng(7)
    return [torch.tensor(rng.integers(0, SMALL["vocab"], PROMPT).astype(np.int32), device="cuda")
            for _ in range(N_MB)]


def reference_tokens(torch, gguf: bool = False, vocab: int = SMALL["vocab"]):
    """Greedy tokens of every sequence from the single-stage Decoder."""
    from dial_cuda.model import Decoder
    dec = Decoder(_cfg(gguf, vocab), n_slots=N_MB, max_seq=PROMPT + STEPS + 8)
    out = []
    for b, p in enumerate(_prompts(torch)):
        tok = dec.prefill(p, slot=b)
        seq = [int(tok.item())]
        for t in range(STEPS):
            o = torch.empty(1, dtype=torch.int32, device="cuda")
            dec.decode_step(tok, torch.tensor([PROMPT + t], dtype=torch.int32, device="cuda"),
                            torch.tensor([b], dtype=torch.int32, device="cuda"), PROMPT + STEPS + 8, o)
            tok = o
            seq.append(int(o.item()))
        out.append(seq)
    return out


def test_single_stage_pipeline_matches_decoder(cuda):
    import torch

    from dial_cuda.model import Stage
    from dial_cuda.pipeline import ModelStageCompute, Pipeline
    ref = reference_tokens(torch)
    cfg = _cfg()
    st = Stage(cfg, 0, cfg.n_layers, n_slots=N_MB, max_seq=PROMPT + STEPS + 8)
    comp = ModelStageCompute(st, N_MB, PROMPT)
    pipe = Pipeline(0, 1, comp, None, N_MB)
    pipe.prefill(_prompts(torch))
    assert [int(t.item()) for t in comp.tokens] == [s[0] for s in ref]
    saved = [t.clone() for t in comp.tokens]
    comp.capture()
    for t, s in zip(comp.tokens, saved):
        t.copy_(s)
    pipe.steps(STEPS - 1)
    pipe.steps(1, host_io=True)
    torch.cuda.synchronize()
    assert [int(t.item()) for t in comp.tokens] == [s[-1] for s in ref]
    assert pipe.host_tokens() == [s[-1] for s in ref]


@pytest.mark.parametrize("gguf", [False, True], ids=["w8a16", "gguf"])
def test_single_stage_micro_batches_match_decoder(cuda, gguf):
    """Batched decode: the 4 sequences as 2 micro-batches of 2 rows (each row its
    own slot and position) give the per-sequence Decoder's tokens."""
    import torch

    from dial_cuda.model import Stage
    from dial_cuda.pipeline import ModelStageCompute, Pipeline
    ref = reference_tokens(torch, gguf)
    cfg = _cfg(gguf)
    R = 2
    st = Stage(cfg, 0, cfg.n_layers, n_slots=N_MB, max_seq=PROMPT + STEPS + 8)
    comp = ModelStageCompute(st, N_MB // R, PROMPT, mb_size=R)
    pipe = Pipeline(0, 1, comp, None, N_MB // R)
    pipe.prefill(_prompts(torch))
    firsts = [int(v) for t in comp.tokens for v in t.tolist()]
    assert firsts == [s[0] for s in ref]
    saved = [t.clone() for t in comp.tokens]
    comp.capture()
    for t, s in zip(comp.tokens, saved):
        t.copy_(s)
    pipe.steps(STEPS - 1)
    pipe.steps(1, host_io=True)
    torch.cuda.synchronize()
    assert [int(v) for t in comp.tokens for v in t.tolist()] == [s[-1] for s in ref]
    assert pipe.host_tokens() == [s[-1] for s in ref]


def _two_stage_worker():
    """Body of one rank (run by torchrun): writes this rank's tokens to DIAL_TEST_OUT."""
    import torch

    from dial_cuda.model import Stage, vocab_shards
    from dial_cuda.pipeline import ModelStageCompute, NcclChannel, Pipeline, head_links, init_distributed
    rank, local, world = init_distributed("nccl", timeout_s=60)
    vocab_head = os.environ.get("DIAL_TEST_VOCAB_HEAD") == "1"
    cfg = _cfg(vocab=VOCAB_PARALLEL if vocab_head else SMALL["vocab"])
    half = cfg.n_layers // 2
    a, b = (0, half) if rank == 0 else (half, cfg.n_layers)
    hch = None
    if vocab_head:
        spans = vocab_shards(cfg.vocab, [1, 1])
        st = Stage(cfg, a, b, n_slots=N_MB, max_seq=PROMPT + STEPS + 8, with_head=False,
                   head_rows=spans[rank])
        comp = ModelStageCompute(st, N_MB, PROMPT, vocab_head_stages=world)
        rows = [v1 - v0 for v0, v1 in spans]
        hch = NcclChannel(rank, world, timeout_s=60.0, links=head_links(world, rows))
        ch = NcclChannel(rank, world, timeout_s=60.0)
        pipe = Pipeline(rank, world, comp, ch, N_MB, head_channel=hch, head_rows=rows)
    else:
        st = Stage(cfg, a, b, n_slots=N_MB, max_seq=PROMPT + STEPS + 8)
        comp = ModelStageCompute(st, N_MB, PROMPT)
        ch = NcclChannel(rank, world, timeout_s=60.0)  # the C ABI's stage communicators
        pipe = Pipeline(rank, world, comp, ch, N_MB)
    pipe.prefill(_prompts(torch) if rank == 0 else None, prompt_len=PROMPT)
    firsts = [int(t.item()) for t in comp.tokens]
    saved = [t.clone() for t in comp.tokens]
    comp.capture()
    for t, s in zip(comp.tokens, saved):
        t.copy_(s)
    pipe.steps(STEPS)
    torch.cuda.synchronize()
    last = [int(t.item()) for t in comp.tokens]
    pipe.finish()
    torch.cuda.synchronize()
    after = [int(t.item()) for t in comp.tokens]
    ch.close()
    if hch is not None:
        hch.close()
    import torch.distributed as dist
    dist.barrier()
    with open(os.path.join(os.environ["DIAL_TEST_OUT"], f"rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "firsts": firsts, "last": last, "after_finish": after}, f)
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


VOCAB_PARALLEL = 8192  # two halves of 256 GEMV tiles each


@pytest.mark.parametrize("vocab_head", [False, True], ids=["head-last", "head-vocab-parallel"])
def test_two_stage_pipeline_matches_single_gpu(cuda, tmp_path, vocab_head):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ref = reference_tokens(torch, vocab=VOCAB_PARALLEL if vocab_head else SMALL["vocab"])
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", DIAL_TEST_OUT=str(tmp_path),
               DIAL_TEST_VOCAB_HEAD="1" if vocab_head else "0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.abspath(__file__)]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert out.returncode == 0, out.stderr[-3000:]
    res = {r: json.loads((tmp_path / f"rank{r}.json").read_text()) for r in (0, 1)}
    assert res[0]["firsts"] == [s[0] for s in ref]   # prefill tokens came back to stage 0
    if not vocab_head:
        assert res[1]["last"] == [s[-1] for s in ref]    # last step's tokens on the last stage
    assert res[0]["after_finish"] == [s[-1] for s in ref]  # and, after finish(), on stage 0


if __name__ == "__main__":  # a rank of the two-stage test
    sys.path.insert(0, os.path.join(ROOT, "dial-8b-orin_b200"))
    _two_stage_worker()
