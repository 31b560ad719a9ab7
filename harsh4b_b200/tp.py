"""Tensor-parallel batch-1 decode over NCCL (one process per GPU).

Partitioning (g ranks; g divides the q heads, the kv heads, the MLP width /
4 and the vocabulary):

* q, k, v rows: rank r owns q heads [r*hq, (r+1)*hq) and kv heads
  [r*hk, (r+1)*hk), so attention and its KV cache stay local;
* o_proj along K (its input is the local heads), down_proj along K (its
  input is the local MLP slice): each rank quantises its slice with the
  GLOBAL activation scale (an all-reduce MAX of the local absmax, one float)
  and produces int32 row sums for all H rows, which an all-reduce SUM adds
  exactly (integers, order-free); every rank then applies the residual
  epilogue to its replicated x;
* gate/up rows: rank r owns MLP units [r*I/g, (r+1)*I/g), so SwiGLU is local;
* LM head rows: rank r owns vocabulary rows [r*V/g, (r+1)*V/g); the greedy
  token is the best (value, global index) over the ranks (all-gather);
* embedding, RMSNorm, residual stream: replicated.

Each rank's slice is itself a valid smaller model (hq heads, hk kv heads,
I/g MLP width, a V/g-row LM head), built by :func:`shard_checkpoint`, so the
single-GPU kernels run it unchanged; only the o/down epilogues move behind
the reductions. Because the sums are exact and the scales are the global
ones, the logits equal the single-GPU decode's bit for bit.
"""
from __future__ import annotations

from dataclasses import replace

import numpy as np

from .cache import Checkpoint, projection_names


def shard_sizes(config: dict, world: int) -> dict:
    heads, kv_heads = int(config["num_attention_heads"]), int(config["num_key_value_heads"])
    inter, vocab = int(config["intermediate_size"]), int(config["vocab_size"])
    if heads % world or kv_heads % world or inter % (4 * world) or vocab % world:
        raise ValueError(f"{world} ranks do not divide heads {heads}, kv heads {kv_heads}, "
                         f"MLP width {inter} (in blocks of 4) and vocabulary {vocab}")
    return {"heads": heads // world, "kv_heads": kv_heads // world, "intermediate": inter // world,
            "vocab": vocab // world}


def shard_checkpoint(checkpoint: Checkpoint, rank: int, world: int) -> Checkpoint:
    """Rank `rank`'s slice as a smaller model. Its embedding/LM-head table is
    the rank's vocabulary rows; the full table stays with the caller for the
    embedding lookup."""
    config = checkpoint.config
    part = shard_sizes(config, world)
    d = int(config["head_dim"])
    qr = slice(rank * part["heads"] * d, (rank + 1) * part["heads"] * d)
    kr = slice(rank * part["kv_heads"] * d, (rank + 1) * part["kv_heads"] * d)
    ir = slice(rank * part["intermediate"], (rank + 1) * part["intermediate"])
    vr = slice(rank * part["vocab"], (rank + 1) * part["vocab"])
    projections = {}
    for name in projection_names(config):
        weights, scales = checkpoint.projections[name]
        kind = name.rsplit(".", 1)[1]
        if kind == "q_proj":
            projections[name] = (weights[qr], scales[qr])
        elif kind in ("k_proj", "v_proj"):
            projections[name] = (weights[kr], scales[kr])
        elif kind == "o_proj":  # K slice: packed bytes hold two columns
            projections[name] = (np.ascontiguousarray(weights[:, qr.start // 2:qr.stop // 2]), scales)
        elif kind in ("gate_proj", "up_proj"):
            projections[name] = (weights[ir], scales[ir])
        elif kind == "down_proj":
            projections[name] = (np.ascontiguousarray(weights[:, ir.start // 2:ir.stop // 2]), scales)
        else:
            raise ValueError(f"unexpected projection {name}")
    sub = dict(config, num_attention_heads=part["heads"], num_key_value_heads=part["kv_heads"],
               intermediate_size=part["intermediate"], vocab_size=part["vocab"])
    return replace(checkpoint, config=sub, projections=projections,
                   embedding=np.ascontiguousarray(checkpoint.embedding[vr]),
                   embedding_scales=np.ascontiguousarray(checkpoint.embedding_scales[vr]),
                   norms=dict(checkpoint.norms))


def global_argmax(values: np.ndarray, indices: np.ndarray) -> int:
    """Best (value, index) over the ranks' local winners: the largest value,
    the smallest global index among equal values (numpy argmax semantics)."""
    best = np.max(values)
    return int(np.min(indices[values == best]))


class TensorParallelQwen:
    """This rank's slice of a g-way tensor-parallel decode (see the module
    docstring). All ranks call forward_token with the same token; each
    returns the greedy token of the full vocabulary and its own logits slice
    (rows [vocab_offset, vocab_offset + V/g)). The process group must use the
    nccl backend, one process per GPU."""

    def __init__(self, checkpoint: Checkpoint, group=None, *, kv_dtype: str = "float16", device=None,
                 attn_splits: int = 16):
        import torch
        import torch.distributed as dist

        from .model import CudaQwen

        self.torch, self.dist, self.group = torch, dist, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        shard = shard_checkpoint(checkpoint, self.rank, self.world)
        self.model = CudaQwen.from_checkpoint(shard, kv_dtype=kv_dtype, device=self.device, attn_splits=attn_splits,
                                              mode="chain")
        self.table = torch.from_numpy(checkpoint.embedding).to(self.device)
        self.table_scales = torch.from_numpy(checkpoint.embedding_scales).to(self.device)
        self.vocab = int(checkpoint.config["vocab_size"])
        self.vocab_offset = self.rank * self.model.vocab
        self.acc = torch.zeros(self.model.hidden, dtype=torch.int32, device=self.device)
        self._best = torch.zeros(2, dtype=torch.float64, device=self.device)
        self._gather = [torch.zeros(2, dtype=torch.float64, device=self.device) for _ in range(self.world)]

    def new_state(self, capacity: int):
        return self.model.new_state(capacity)

    def _stage(self, state, stage: int, layer: int = 0) -> None:
        import ctypes

        from ._lib import check, lib

        check(lib().h4b_decode_stage(ctypes.byref(self.model.desc), ctypes.byref(state.desc), stage, layer,
                                     self.torch.cuda.current_stream(self.device).cuda_stream), "h4b_decode_stage")

    def forward_token(self, token_id: int, state):
        """One token on every rank; returns (greedy token, local logits slice)."""
        from . import ops

        torch, dist, m = self.torch, self.dist, self.model
        if state.position >= state.capacity:
            raise ValueError("decode state capacity exhausted")
        if not 0 <= int(token_id) < self.vocab:
            raise ValueError(f"token ID {token_id} is outside the vocabulary")
        state.absmax.zero_()
        state.argmax_key.zero_()
        state.token_dev.fill_(int(token_id))
        ops.embedding(state.token_dev, self.table, self.table_scales, out=state.x)
        H, I = m.hidden, m.intermediate
        for l in range(m.n_layers):
            self._stage(state, 1, l)  # qkv rows of the local heads (RMSNorm + quantise fused)
            self._stage(state, 2, l)  # local attention; absmax[2l] = local max of attended
            amax = state.absmax[2 * l:2 * l + 1]
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
            ops.int4_gemv_absmax(state.attended, amax, m.w_o[l], m.s_o[l], self.acc)
            dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
            ops.residual_acc(state.x, self.acc, amax, m.s_o[l])
            self._stage(state, 4, l)  # local gate/up + SwiGLU; absmax[2l+1] = local max of act
            amax = state.absmax[2 * l + 1:2 * l + 2]
            dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
            ops.int4_gemv_absmax(state.act, amax, m.w_down[l], m.s_down[l], self.acc)
            dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
            ops.residual_acc(state.x, self.acc, amax, m.s_down[l])
        self._stage(state, 6)  # local LM head rows + local argmax key
        self._stage(state, 7)  # next_token (local index) and position += 1
        state.position += 1
        local = int(state.next_token_dev.item())
        self._best[0] = state.logits[local].to(torch.float64)
        self._best[1] = float(local + self.vocab_offset)
        dist.all_gather(self._gather, self._best, group=self.group)
        pairs = torch.stack(self._gather).cpu().numpy()
        token = global_argmax(pairs[:, 0], pairs[:, 1].astype(np.int64))
        return token, state.logits
