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

Prefill (:meth:`TensorParallelQwen.prefill`) shards the same way with M
prompt rows at a time: every rank runs its slice's GEMMs over all rows
(h4b_prefill_tp_stage), the per-row absmax of the o / down inputs is reduced
with MAX over the ranks ([M] floats) and their int32 row sums with SUM
([M][H] int32, 21 MB at M = 2048), both as NCCL all-reduces.

The exchanges run either as single-kernel one-shot transfers over NVLink
peer memory (comm="p2p", csrc/tp.cu: the absmax MAX, the int32 SUM fused
with the residual epilogue, the greedy candidates) or as NCCL collectives
(comm="nccl"); both give the same bits.

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
                 attn_splits: int = 16, comm: str = "p2p"):
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
        self._gathered = torch.zeros(2 * self.world, dtype=torch.float64, device=self.device)
        self._token_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._graphs = {}
        if comm not in ("p2p", "nccl"):
            raise ValueError("comm must be 'p2p' or 'nccl'")
        self.comm, self._own, self._peers, self.group_desc = comm, None, [], None
        if comm == "p2p":
            self._open_peer_buffers()

    def _open_peer_buffers(self) -> None:
        """Allocates this rank's receive buffer, exchanges IPC handles over the
        process group and maps every peer's buffer (h4b_tp_group)."""
        import ctypes

        from ._lib import TpGroupDesc, check, lib

        torch, dist = self.torch, self.dist
        capacity = max(self.model.hidden, 2)
        nbytes = int(lib().h4b_tp_buffer_bytes(self.world, capacity))
        check(nbytes if nbytes < 0 else 0, "h4b_tp_buffer_bytes")
        own, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            check(lib().h4b_ipc_alloc(nbytes, ctypes.byref(own), handle), "h4b_ipc_alloc")
            self._own = own.value
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=self.group)
            buffers = (ctypes.c_void_p * 8)()
            for r in range(self.world):
                if r == self.rank:
                    buffers[r] = self._own
                    continue
                peer = ctypes.c_void_p()
                check(lib().h4b_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(peer)),
                      "h4b_ipc_open")
                self._peers.append(peer.value)
                buffers[r] = peer.value
        self._generation = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.group_desc = TpGroupDesc(self.world, self.rank, capacity, buffers, self._generation.data_ptr())

    def close(self) -> None:
        """Releases the graphs and the peer mappings (before the process group
        is destroyed; every rank calls it)."""
        from ._lib import lib

        self.release_graphs()
        self.torch.cuda.synchronize(self.device)
        with self.torch.cuda.device(self.device):
            for peer in self._peers:
                lib().h4b_ipc_close(peer)
            self._peers = []
            if self._own is not None:
                self.dist.barrier(group=self.group)  # no peer writes into it any more
                lib().h4b_ipc_free(self._own)
                self._own = None

    def new_state(self, capacity: int):
        return self.model.new_state(capacity)

    def _stage(self, state, stage: int, layer: int = 0) -> None:
        import ctypes

        from ._lib import check, lib

        check(lib().h4b_decode_stage(ctypes.byref(self.model.desc), ctypes.byref(state.desc), stage, layer,
                                     self.torch.cuda.current_stream(self.device).cuda_stream), "h4b_decode_stage")

    def forward_token(self, token_id: int, state, graph: bool = False):
        """One token on every rank; returns (greedy token, local logits slice).
        graph=True replays the whole token (kernels and collectives) as one
        CUDA graph per state, captured on first use; the host then only
        copies the token id in and the ranks' candidates out."""
        if state.position >= state.capacity:
            raise ValueError("decode state capacity exhausted")
        if not 0 <= int(token_id) < self.vocab:
            raise ValueError(f"token ID {token_id} is outside the vocabulary")
        self._token_host[0] = int(token_id)
        state.token_dev.copy_(self._token_host, non_blocking=True)
        if graph:
            cuda_graph = self._graphs.get(id(state))
            if cuda_graph is None:
                cuda_graph = self._capture(state)
            cuda_graph.replay()
        else:
            self._token_body(state)
        state.position += 1
        pairs = self._gathered.cpu().numpy().reshape(self.world, 2)  # waits for the token
        token = global_argmax(pairs[:, 0], pairs[:, 1].astype(np.int64))
        return token, state.logits

    def _capture(self, state):
        """Captures _token_body for `state` (the token id is read from
        state.token_dev, the position from the device, so replays advance)."""
        torch, dist = self.torch, self.dist
        if self.comm == "nccl":  # the communicators must exist before a capture
            probe = torch.zeros(2, dtype=torch.float64, device=self.device)
            dist.all_reduce(probe[:1], op=dist.ReduceOp.MAX, group=self.group)
            dist.all_reduce(self.acc.new_zeros(1), op=dist.ReduceOp.SUM, group=self.group)
            dist.all_gather_into_tensor(self._gathered.clone(), probe, group=self.group)
        torch.cuda.synchronize(self.device)
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self._token_body(state)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self._graphs[id(state)] = graph
        return graph

    def release_graphs(self) -> None:
        """Drops the captured graphs (they hold NCCL work: release them before
        the process group is destroyed)."""
        self._graphs.clear()

    def _token_body(self, state) -> None:
        """Every kernel and exchange of one token, on the current stream."""
        from . import ops

        torch, dist, m = self.torch, self.dist, self.model
        state.absmax.zero_()
        state.argmax_key.zero_()
        ops.embedding(state.token_dev, self.table, self.table_scales, out=state.x)
        for l in range(m.n_layers):
            self._stage(state, 1, l)  # qkv rows of the local heads (RMSNorm + quantise fused)
            self._stage(state, 2, l)  # local attention; absmax[2l] = local max of attended
            self._k_split(state, state.attended, state.absmax[2 * l:2 * l + 1], m.w_o[l], m.s_o[l])
            self._stage(state, 4, l)  # local gate/up + SwiGLU; absmax[2l+1] = local max of act
            self._k_split(state, state.act, state.absmax[2 * l + 1:2 * l + 2], m.w_down[l], m.s_down[l])
        self._stage(state, 6)  # local LM head rows + local argmax key
        self._stage(state, 7)  # next_token (local index) and position += 1
        if self.comm == "p2p":
            self._p2p("h4b_tp_gather_best", state.logits.data_ptr(), state.next_token_dev.data_ptr(),
                      self.vocab_offset, self._gathered.data_ptr())
            return
        local = state.next_token_dev.to(torch.int64)
        self._best[0:1].copy_(state.logits.index_select(0, local))
        self._best[1:2].copy_(local + self.vocab_offset)
        dist.all_gather_into_tensor(self._gathered, self._best, group=self.group)

    def prefill(self, token_ids, state, max_tokens: int = 2048, attn_splits: int = 1, attention: str = "tensor"):
        """Feed a prompt on every rank (all ranks pass the same ids): the
        sharded h4b_prefill_tp_stage sequence with NCCL all-reduces of the
        per-row absmax (MAX) and of the o / down int32 row sums (SUM)
        between the stages. Returns (greedy token, local logits slice) of the
        last prompt row. With attention="exact" the state then stands where
        forward_token over the same ids with `attn_splits` splits per prompt
        query leaves it; "tensor" is CudaQwen.prefill's tensor-core attention."""
        import ctypes

        from ._lib import check, lib
        from .model import PREFILL_ATTENTION, PrefillScratch

        if attention not in PREFILL_ATTENTION:
            raise ValueError(f"attention must be one of {sorted(PREFILL_ATTENTION)}")

        torch, dist, m = self.torch, self.dist, self.model
        ids = np.asarray([int(t) for t in token_ids], dtype=np.int32)
        if ids.size == 0:
            raise ValueError("empty prompt")
        if state.position + ids.size > state.capacity:
            raise ValueError("decode state capacity exhausted")
        if ids.min() < 0 or ids.max() >= self.vocab:
            raise ValueError("token ID outside the vocabulary")
        rows = min(int(max_tokens), int(ids.size))
        scratch = m._prefill_scratch
        if scratch is None or scratch.max_tokens < rows or scratch.splits != int(attn_splits):
            scratch = m._prefill_scratch = PrefillScratch(m, rows, int(attn_splits))
        scratch.desc.attn_kernel = PREFILL_ATTENTION[attention]
        absmax = torch.empty(scratch.max_tokens, dtype=torch.float32, device=self.device)
        acc = torch.empty(scratch.max_tokens, m.hidden, dtype=torch.int32, device=self.device)
        stream = torch.cuda.current_stream(self.device)

        def stage(count, layer, index):
            check(lib().h4b_prefill_tp_stage(ctypes.byref(m.desc), ctypes.byref(state.desc), ctypes.byref(scratch.desc),
                                             count, layer, index, self.table.data_ptr(), self.table_scales.data_ptr(),
                                             self.vocab, absmax.data_ptr(), acc.data_ptr(), stream.cuda_stream),
                  "h4b_prefill_tp_stage")

        MAX, SUM = dist.ReduceOp.MAX, dist.ReduceOp.SUM
        for start in range(0, ids.size, scratch.max_tokens):
            part = ids[start:start + scratch.max_tokens]
            n = int(part.size)
            scratch.tokens[:n].copy_(torch.from_numpy(part))
            stage(n, 0, 0)
            for layer in range(m.n_layers):
                stage(n, layer, 1)
                dist.all_reduce(absmax[:n], op=MAX, group=self.group)
                stage(n, layer, 2)
                dist.all_reduce(acc[:n], op=SUM, group=self.group)
                stage(n, layer, 3)
                dist.all_reduce(absmax[:n], op=MAX, group=self.group)
                stage(n, layer, 4)
                dist.all_reduce(acc[:n], op=SUM, group=self.group)
                stage(n, layer, 5)
            stage(n, 0, 6)
            state.position += n
        local = state.next_token_dev.to(torch.int64)
        self._best[0:1].copy_(state.logits.index_select(0, local))
        self._best[1:2].copy_(local + self.vocab_offset)
        dist.all_gather_into_tensor(self._gathered, self._best, group=self.group)
        pairs = self._gathered.cpu().numpy().reshape(self.world, 2)
        token = global_argmax(pairs[:, 0], pairs[:, 1].astype(np.int64))
        return token, state.logits

    def _p2p(self, name: str, *args) -> None:
        import ctypes

        from ._lib import check, lib

        stream = self.torch.cuda.current_stream(self.device).cuda_stream
        check(getattr(lib(), name)(ctypes.byref(self.group_desc), *args, stream), name)

    def _k_split(self, state, values, amax, weights, scales) -> None:
        """A K-split projection (o or down): the global quantisation scale, this
        rank's int32 row sums, their exact sum over the ranks, the residual."""
        from . import ops

        dist, H = self.dist, self.model.hidden
        if self.comm == "p2p":
            self._p2p("h4b_tp_allreduce_max", amax.data_ptr())
            ops.int4_gemv_absmax(values, amax, weights, scales, self.acc)
            self._p2p("h4b_tp_allreduce_sum_residual", self.acc.data_ptr(), state.x.data_ptr(), amax.data_ptr(),
                      scales.data_ptr(), H)
            return
        dist.all_reduce(amax, op=dist.ReduceOp.MAX, group=self.group)
        ops.int4_gemv_absmax(values, amax, weights, scales, self.acc)
        dist.all_reduce(self.acc, op=dist.ReduceOp.SUM, group=self.group)
        ops.residual_acc(state.x, self.acc, amax, scales)
