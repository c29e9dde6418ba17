"""GPU (2 devices): the layer-range pipeline over NCCL gives the tokens of
the single-GPU engine, bit for bit (the same kernels run on the same layers;
only the hand-off of x[dim] between stages is new) — through the library's
own stage transport (leap_pp_*) and through torch.distributed.

Skipped unless two CUDA devices are visible.  Each stage is its own process
(one per GPU) with a short process-group timeout.
"""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stage(rank, world, port, quantized, q, comm_kind):
    import torch.distributed as dist

    from leap_b200 import ModelConfig, Transformer
    from leap_b200.pipeline import NativeComm, PipelineStage, TorchComm, stage_range
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        cfg = ModelConfig(1024, 2816, 6, 16, 4, 4096, 512)
        prompt = [int(t) for t in torch.randint(0, cfg.vocab_size, (45,),
                                                generator=torch.Generator().manual_seed(5))]
        lb, le = stage_range(cfg.n_layers, rank, world)
        with Transformer.synthetic(cfg, quantized, seed=11, device=rank, layer_range=(lb, le),
                                   max_chunk=16) as eng:
            eng.bind_torch_stream()
            comm = NativeComm(rank, world, rank, 30000) if comm_kind == "native" else TorchComm()
            st = PipelineStage(eng, cfg.dim, dev, max_chunk=16, comm=comm)
            toks = st.generate(prompt, 40, chunk=16)
            torch.cuda.synchronize()
            comm.close()
        want = None
        if rank == 0:
            with Transformer.synthetic(cfg, quantized, seed=11, device=rank, max_chunk=16) as full:
                full.bind_torch_stream()
                one = PipelineStage(full, cfg.dim, dev, max_chunk=16, rank=0, world=1)
                want = one.generate(prompt, 40, chunk=16)
        q.put((rank, "ok", toks, want))
    except Exception as exc:
        q.put((rank, "error", repr(exc)[:300], None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("comm_kind", ["native", "torch"])
@pytest.mark.parametrize("quantized", [False, True])
def test_two_stage_pipeline_matches_single_gpu(cuda, quantized, comm_kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stage, args=(r, 2, port, quantized, q, comm_kind)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, status, toks, want = q.get(timeout=300)
        res[r] = (status, toks, want)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    assert res[1][1] is None
    assert len(res[0][1]) == 40
    assert res[0][1] == res[0][2]
