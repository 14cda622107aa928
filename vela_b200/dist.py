"""Box-level partition of independent inferences over the GPUs of one node (no collectives on the data path).

Every inference depends only on its 32-byte seed, the read-only model and the prompt context, so a box
runs one process per GPU, each with its own model copy and lanes, on a disjoint block of seeds
(the reference's multi-GPU miner: src/main.cpp:117-123, tests/multi_gpu.py:17-24).  The only
cross-rank traffic is host bookkeeping: a barrier around timed regions, the maximum of the ranks'
times and a comparison of x0 digests, all through torch.distributed (NCCL on GPUs, gloo on CPU).
"""
import hashlib
import struct

import numpy as np


def seed_block(rank, lane, step, batch, salt=b"vela-b200-bench"):
    """seeds [batch, 32] uint8 of (rank, lane, step): SHA-256 of salt | rank | lane | step | index, disjoint across ranks"""
    out = np.empty((batch, 32), np.uint8)
    for b in range(batch):
        out[b] = np.frombuffer(hashlib.sha256(salt + struct.pack("<4Q", rank, lane, step, b)).digest(), np.uint8)
    return out


def golden_seeds(batch):
    """the parity seeds: seed_b = SHA-256("vela-b200" | b), b < batch (same on every rank)"""
    return np.stack([np.frombuffer(hashlib.sha256(b"vela-b200" + bytes([b])).digest(), np.uint8) for b in range(batch)])


def max_over_ranks(value, device=None):
    """max of a float over all ranks (the value itself when torch.distributed is not initialised)"""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def digests_agree(digest, device=None):
    """True on every rank iff all ranks hold the same 32-byte digest"""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return True
    mine = torch.tensor(list(digest), dtype=torch.int64, device=device)
    lo, hi = mine.clone(), mine.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    return bool(torch.equal(lo, hi))
