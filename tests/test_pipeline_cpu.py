"""CPU: the pipeline schedule (leap_b200.pipeline) as gloo ranks.

A small deterministic model stands in for the engine: an embedding table,
per-layer maps that also read the layer's own cache of earlier positions
(so a stage that saw the wrong positions, or the wrong order, changes the
tokens), and an argmax head.  World sizes 2 and 3, over ragged prompt chunks,
must produce exactly the tokens of the same model run as one stage.  A stage
that fails before its first receive makes its neighbours fail with an error
within the process group timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from leap_b200.pipeline import PipelineStage, stage_range

DIM, VOCAB, LAYERS, SEQ = 16, 50, 6, 128


class ToyStage:
    """Layers [lb, le) of the toy model, with the Transformer stage API."""

    def __init__(self, lb, le, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.emb = torch.randn(VOCAB, DIM, generator=g, dtype=torch.float64)
        self.w = [torch.randn(DIM, DIM, generator=g, dtype=torch.float64) / DIM ** 0.5
                  for _ in range(LAYERS)]
        self.cls = torch.randn(VOCAB, DIM, generator=g, dtype=torch.float64)
        self.lb, self.le = lb, le
        self.cache = {l: torch.zeros(SEQ, DIM, dtype=torch.float64) for l in range(lb, le)}
        self.seen = {l: -1 for l in range(lb, le)}

    def embed(self, tokens, x):
        x.copy_(self.emb[torch.as_tensor(list(tokens))].to(x.dtype))

    def embed_device(self, tok, x):
        x.copy_(self.emb[tok.long()].to(x.dtype))

    def layers(self, pos0, x):
        h = x.to(torch.float64)
        for l in range(self.lb, self.le):
            for r in range(h.shape[0]):
                pos = pos0 + r
                assert pos == self.seen[l] + 1, "positions must arrive in order"
                self.seen[l] = pos
                ctx = self.cache[l][:pos].mean(0) if pos else torch.zeros(DIM, dtype=torch.float64)
                h[r] = torch.tanh(h[r] @ self.w[l] + 0.5 * ctx + 0.01 * pos)
                self.cache[l][pos] = h[r]
        x.copy_(h.to(x.dtype))

    def head(self, x, logits, token):
        lg = self.cls @ x.reshape(-1).to(torch.float64)
        if logits is not None:
            logits.copy_(lg.to(logits.dtype))
        if token is not None:
            token.fill_(int(torch.argmax(lg)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _single_stage_tokens(prompt, steps, chunk):
    st = PipelineStage(ToyStage(0, LAYERS), DIM, "cpu", max_chunk=chunk, rank=0, world=1)
    return st.generate(prompt, steps, chunk)


def _worker(rank, world, port, prompt, steps, chunk, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        if rank == fail_rank:
            raise RuntimeError("stage failed before its first receive")
        lb, le = stage_range(LAYERS, rank, world)
        st = PipelineStage(ToyStage(lb, le), DIM, "cpu", max_chunk=chunk)
        toks = st.generate(prompt, steps, chunk)
        q.put((rank, "ok", toks))
    except Exception as exc:  # reported to the test, which asserts on it
        q.put((rank, "error", type(exc).__name__ + ": " + str(exc)[:200]))
    finally:
        if rank != fail_rank:
            dist.destroy_process_group()


def _run(world, prompt, steps, chunk, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, prompt, steps, chunk, q, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, val = q.get(timeout=120)
        out[r] = (status, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_stage_ranges_cover_layers():
    for L in (1, 6, 22, 32, 80):
        for N in (1, 2, 3, 4, 8):
            if N > L:
                with pytest.raises(ValueError):
                    stage_range(L, 0, N)
                continue
            rs = [stage_range(L, i, N) for i in range(N)]
            assert rs[0][0] == 0 and rs[-1][1] == L
            assert all(a[1] == b[0] and a[0] < a[1] for a, b in zip(rs, rs[1:]))
    assert stage_range(80, 3, 8) == (30, 40)


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_matches_single_stage(world):
    prompt = [3, 14, 15, 9, 26, 5, 35, 8, 9, 7, 9, 32, 38, 46, 26]
    steps, chunk = 12, 4  # ragged: 4 + 4 + 4 + 3
    want = _single_stage_tokens(prompt, steps, chunk)
    out = _run(world, prompt, steps, chunk)
    assert out[0] == ("ok", want)
    for r in range(1, world):
        assert out[r] == ("ok", None)


def test_failed_stage_surfaces_as_error():
    out = _run(2, [1, 2, 3], 4, 2, fail_rank=1)
    assert out[1][0] == "error"
    assert out[0][0] == "error", out  # rank 0's send/recv ends with an error, not a hang
