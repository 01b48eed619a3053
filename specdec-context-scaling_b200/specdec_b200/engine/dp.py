"""Data-parallel SpecDec over the GPUs of one node: sequences are independent, so rank
r takes a contiguous block of them, builds the same seeded random-init models, and
runs prefill + decode with no collective; one all-gather of the emitted tokens (and
a max-reduce of the per-rank times) at the end is the only communication.

Works with any torch.distributed backend: NCCL on GPUs, gloo in the CPU tests.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous block; block sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank outside the world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def synthetic_prompts(total: int, prompt_len: int, vocab: int, seed: int) -> torch.Tensor:
    """(total, prompt_len) int32 uniform-random token ids, identical on every rank."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (total, prompt_len), generator=g, dtype=torch.int64).to(torch.int32)


def gather_rows(local: torch.Tensor, total: int, world: int, group=None) -> torch.Tensor:
    """All-gather of each rank's block of rows (blocks from shard_bounds) into (total, ...)."""
    import torch.distributed as dist

    if world == 1:
        return local
    per = -(-total // world)  # equal-size buffers for all_gather; rows past a block are padding
    buf = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    rows = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        rows.append(parts[r][:e - s])
    return torch.cat(rows, dim=0)


def max_over_ranks(x: float, world: int, device) -> float:
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def check_shardable(total_seqs: int, world: int) -> None:
    """Every rank must get at least one sequence: an empty shard cannot build its engine,
    and a rank that fails alone would leave the others waiting in the final collectives.
    The check depends only on arguments every rank shares, so all ranks raise together,
    before any collective."""
    if total_seqs < world:
        raise ValueError(f"{total_seqs} sequences cannot be sharded over {world} ranks (at least one per rank)")


@dataclass
class DPResult:
    tokens: torch.Tensor      # (total, max_new): gathered from every rank
    decode_s: float           # max over ranks of the decode time
    prefill_s: float          # max over ranks
    rounds: int
    acceptance: float         # mean accepted candidates per round and sequence (local)
    local_seqs: int


def run_specdec_dp(target_cfg, draft_cfg, *, total_seqs: int, prompt_len: int, max_new: int, k: int = 4,
                   seed: int = 0, world: int = 1, rank: int = 0, target_v: str = "bf16", chunk: int = 4,
                   barrier=None, draft_is_target: bool = False) -> DPResult:
    """One data-parallel SpecDec job on this rank's GPU (weights from ``seed``).  The
    decode time is the device time of the round-graph replays (CUDA events).
    ``draft_is_target``: the draft runs the target's weights (``draft_cfg`` is ignored), so
    nearly every candidate is accepted -- the full-accept path of every round."""
    from .model import PagedModel
    from .specdec import SpecDecEngine

    check_shardable(total_seqs, world)
    dev = torch.device("cuda", torch.cuda.current_device())
    s, e = shard_bounds(total_seqs, world, rank)
    prompts = synthetic_prompts(total_seqs, prompt_len, target_cfg.vocab, seed)[s:e].to(dev)
    if draft_is_target:
        from .model import random_state

        state = random_state(target_cfg, seed + 1, dev)
        target, draft = PagedModel(target_cfg, state, dev), PagedModel(target_cfg, state, dev)
        del state
    else:
        target = PagedModel.random(target_cfg, seed + 1, dev)
        draft = PagedModel.random(draft_cfg, seed + 2, dev)
    eng = SpecDecEngine(target, draft, e - s, prompt_len, max_new, k=k, target_v=target_v)
    eng.capture()  # warm-up round + graph capture on the empty state; prefill resets it
    sync = barrier or (lambda: None)
    torch.cuda.synchronize()
    sync()
    t0 = time.perf_counter()
    eng.prefill(prompts, chunk=chunk)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    rounds = eng.decode()
    ev1.record()
    torch.cuda.synchronize()
    dec = ev0.elapsed_time(ev1) / 1e3
    toks = gather_rows(eng.tokens().contiguous(), total_seqs, world)
    return DPResult(toks, max_over_ranks(dec, world, dev), max_over_ranks(t1 - t0, world, dev), rounds,
                    eng.acceptance(), e - s)
