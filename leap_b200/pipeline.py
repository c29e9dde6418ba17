"""Layer-range pipeline stages: one process per GPU, activations handed
between consecutive stages with point-to-point sends over NCCL.

The reference splits a model layer-wise across a ring of devices: the master
runs layers [0, split_layer) and the workers the rest, and each hop carries a
PacketHeader {pos, flags} plus x[dim] over TCP/UDP or its kernel-module
transport (src/inference/Transformer.h:17-23, FloatTransformer.cpp:751-797
master forward, :800-946 worker_loop).  Inside one B200 box the same split
runs as N stages, one per GPU:

* stage i of N owns layers [floor(L*i/N), floor(L*(i+1)/N)) and their KV
  cache; stage 0 also owns the embedding, the last stage the final norm, the
  classifier and the greedy sampler (so only a 4-byte token id goes back to
  stage 0 instead of the reference's round trip of x to the master);
* every stage knows (pos, n) from the shared step schedule, so a hop carries
  only the activation rows x[n][dim];
* a prompt moves in chunks, so stage i works on chunk c while stage i+1
  works on chunk c-1;
* everything is stream-ordered: stage 0 embeds the token the last stage
  sent straight from device memory, and no stage waits on its host between
  decode steps.

The hop goes through a transport object with `send(tensor, dst)` and
`recv(tensor, src)`: `NativeComm` is the library's own stage transport
(`leap_pp_*`, NCCL point-to-point over NVLink, bounded by a timeout and
abortable), `TorchComm` is torch.distributed point-to-point on the default
process group (used by the CPU tests of the schedule, over gloo).  The
engine is anything with the stage operations of `leap_b200.Transformer`
(`embed`, `embed_device`, `layers`, `head` on tensors).
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch
import torch.distributed as dist

__all__ = ["stage_range", "PipelineStage", "StageTimes", "TorchComm", "NativeComm"]


class TorchComm:
    """Point-to-point on torch.distributed's default group."""

    def send(self, t: torch.Tensor, dst: int) -> None:
        dist.send(t, dst=dst)

    def recv(self, t: torch.Tensor, src: int) -> None:
        dist.recv(t, src=src)

    def close(self) -> None:
        pass


class NativeComm:
    """The library's stage transport (leap_pp_*): NCCL point-to-point over
    NVLink, enqueued on the current torch stream.  The 128-byte job id is
    made by rank 0 and handed to the others over the default process group
    (any host channel would do)."""

    def __init__(self, rank: int, world: int, device: int, timeout_ms: int = 60000):
        from ._native import check, lib
        self._lib, self._check = lib(), check
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            check(self._lib.leap_pp_unique_id(uid))
        if world > 1:
            t = torch.frombuffer(bytearray(uid.raw), dtype=torch.uint8).clone()
            if dist.get_backend() == "nccl":
                t = t.cuda(device)
            dist.broadcast(t, src=0)
            uid = ctypes.create_string_buffer(bytes(t.cpu().tolist()), 128)
        self._h = ctypes.c_void_p()
        check(self._lib.leap_pp_init(uid, rank, world, device, timeout_ms, ctypes.byref(self._h)))

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def send(self, t: torch.Tensor, dst: int) -> None:
        self._check(self._lib.leap_pp_send(self._h, dst, ctypes.c_void_p(t.data_ptr()),
                                           t.numel() * t.element_size(), self._stream()))

    def recv(self, t: torch.Tensor, src: int) -> None:
        self._check(self._lib.leap_pp_recv(self._h, src, ctypes.c_void_p(t.data_ptr()),
                                           t.numel() * t.element_size(), self._stream()))

    def abort(self) -> None:
        """End transfers whose peer has gone (the communicator is unusable after)."""
        if self._h:
            self._lib.leap_pp_abort(self._h)

    def close(self) -> None:
        if self._h:
            h, self._h = self._h, None
            self._check(self._lib.leap_pp_destroy(h))


def stage_range(n_layers: int, rank: int, world: int) -> tuple[int, int]:
    """Layers [begin, end) of stage `rank` of `world`: floor(L*i/N)."""
    if not 0 <= rank < world or world > n_layers:
        raise ValueError(f"stage {rank} of {world} for {n_layers} layers")
    return n_layers * rank // world, n_layers * (rank + 1) // world


@dataclasses.dataclass
class StageTimes:
    prefill_s: float = 0.0
    decode_s: float = 0.0


class PipelineStage:
    """One stage of the pipeline (this process's rank in the default group).

    `engine` holds this stage's layer range; `dim` is the model width;
    `device` is where activations live (a CUDA device, or CPU for gloo)."""

    def __init__(self, engine, dim: int, device, max_chunk: int = 512, rank=None, world=None,
                 comm=None):
        self.e = engine
        self.comm = comm if comm is not None else TorchComm()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.first = self.rank == 0
        self.last = self.rank == self.world - 1
        self.device = torch.device(device)
        self.max_chunk = max_chunk
        self.x = torch.empty((max_chunk, dim), dtype=torch.float32, device=self.device)
        self.tok = torch.zeros(1, dtype=torch.int32, device=self.device)

    # -- one hop ---------------------------------------------------------------
    def _rows(self, pos0: int, n: int, tokens=None) -> torch.Tensor:
        """Run positions pos0..pos0+n-1 through this stage; returns x[n]."""
        x = self.x[:n]
        if self.first:
            if tokens is None:
                self.e.embed_device(self.tok, x)
            else:
                self.e.embed(tokens, x)
        else:
            self.comm.recv(x, self.rank - 1)
        self.e.layers(pos0, x)
        if not self.last:
            self.comm.send(x, self.rank + 1)
        return x

    def _token_to_first(self) -> None:
        if self.world == 1:
            return
        if self.last:
            self.comm.send(self.tok, 0)
        elif self.first:
            self.comm.recv(self.tok, self.world - 1)

    # -- the reference's generate loop, split across stages ---------------------
    def prefill(self, prompt, pos0: int = 0, chunk: int | None = None) -> None:
        """Prompt tokens pos0.. into every stage's KV cache; the greedy token
        after the prompt ends up in `self.tok` on stage 0 (and the last)."""
        chunk = min(chunk or self.max_chunk, self.max_chunk)
        prompt = list(prompt)
        x = None
        for c0 in range(0, len(prompt), chunk):
            part = prompt[c0:c0 + chunk]
            x = self._rows(pos0 + c0, len(part), part)
        if self.last:
            self.e.head(x[-1:], None, self.tok)
        self._token_to_first()

    def decode(self, pos: int, steps: int) -> torch.Tensor:
        """`steps` greedy tokens from `self.tok` at position `pos` on; returns
        them on stage 0 (a device tensor; empty on the other stages)."""
        out = torch.empty(steps if self.first else 0, dtype=torch.int32, device=self.device)
        for i in range(steps):
            x = self._rows(pos + i, 1)
            if self.last:
                self.e.head(x, None, self.tok)
            self._token_to_first()
            if self.first:
                out[i:i + 1].copy_(self.tok)
        return out

    def generate(self, prompt, steps: int, chunk: int | None = None):
        """Prompt, then `steps` greedy tokens (the first is the prefill's):
        main.cpp:64-108 at temperature 0.  Returns the tokens on stage 0,
        None elsewhere."""
        prompt = list(prompt)
        self.prefill(prompt, 0, chunk)
        if self.first:
            first = self.tok.clone()
        rest = self.decode(len(prompt), steps - 1) if steps > 1 else None
        if not self.first:
            return None
        toks = [int(first.item())]
        if rest is not None:
            toks += [int(t) for t in rest.cpu().tolist()]
        return toks
