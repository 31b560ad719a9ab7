"""Tensor-parallel decode: the sharding and reduction math (harsh4b_b200.tp)
checked on CPU with two gloo ranks running the oracle's primitives, against
the unsharded oracle bit for bit; and on two GPUs (when present) against the
single-GPU decode."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import oracle  # noqa: E402
from _models import oracle_model  # noqa: E402
from harsh4b_b200.synthetic import synthetic_checkpoint, synthetic_prompt, tiny_config  # noqa: E402
from harsh4b_b200.tp import global_argmax, shard_checkpoint, shard_sizes  # noqa: E402

SEED, STEPS = 31, 6


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _quantize_with_max(values, global_max):
    """quantize_activation with the absmax of the whole (sharded) vector: the
    oracle's own routine over the local values plus a sentinel equal to it."""
    padded = np.append(values, np.float32(global_max)).astype(np.float32)
    q = np.empty(padded.size, dtype=np.int8)
    scale = oracle.quantize_activation(padded, q)
    return q[:-1].copy(), scale


def _allreduce(array, op):
    t = torch.from_numpy(np.ascontiguousarray(array))
    dist.all_reduce(t, op=op)
    return t.numpy()


def _tp_oracle_rank(rank, world, port, results):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ck = synthetic_checkpoint(tiny_config(), seed=SEED)
        full = oracle_model(ck, attn_splits=2)
        part = oracle_model(shard_checkpoint(ck, rank, world), attn_splits=2)
        st = part.new_state(32)
        prompt = synthetic_prompt(ck.config, STEPS, seed=SEED)
        outs = []
        for token in prompt:
            x = st.x
            full.embedding_into(int(token), x)
            q_end, k_end = part.q_size, part.q_size + part.kv_size
            for index, layer in enumerate(part.layers):
                part.kernel.rmsnorm_into(x, layer.input_norm, st.normalized, part.eps)
                q8, s = part.quantize(st.normalized, st)
                part.project(layer.qkv, q8, s, st.qkv)
                q = st.qkv[:q_end].reshape(part.heads, part.head_dim)
                k = st.qkv[q_end:k_end].reshape(part.kv_heads, part.head_dim)
                v = st.qkv[k_end:].reshape(part.kv_heads, part.head_dim)
                part.qk_norm(q, layer.q_norm)
                part.qk_norm(k, layer.k_norm)
                part.rope(q, st.position)
                part.rope(k, st.position)
                st.keys[index, st.position] = k
                st.values[index, st.position] = v
                part.attention(st, index, q)
                g = _allreduce(np.array([np.abs(st.attended).max()], np.float32), dist.ReduceOp.MAX)[0]
                q8, s = _quantize_with_max(st.attended, g)
                _, acc = oracle.int4_gemv(q8, layer.o.weights, layer.o.scales, s)
                acc = _allreduce(acc, dist.ReduceOp.SUM)
                x += (acc.astype(np.float32) * np.float32(s)) * layer.o.scales
                part.kernel.rmsnorm_into(x, layer.post_norm, st.normalized, part.eps)
                q8, s = part.quantize(st.normalized, st)
                part.project(layer.gate_up, q8, s, st.gate_up)
                oracle.library().oracle_silu_mul(oracle._ptr(st.gate_up[:part.intermediate]),
                                                 oracle._ptr(st.gate_up[part.intermediate:]),
                                                 oracle._ptr(st.activated), part.intermediate)
                g = _allreduce(np.array([np.abs(st.activated).max()], np.float32), dist.ReduceOp.MAX)[0]
                q8, s = _quantize_with_max(st.activated, g)
                _, acc = oracle.int4_gemv(q8, layer.down.weights, layer.down.scales, s)
                acc = _allreduce(acc, dist.ReduceOp.SUM)
                x += (acc.astype(np.float32) * np.float32(s)) * layer.down.scales
            part.kernel.rmsnorm_into(x, part.final_norm, st.normalized, part.eps)
            q8, s = part.quantize(st.normalized, st)
            part.project(part.lm_head, q8, s, st.logits)
            st.position += 1
            gathered = [torch.zeros(st.logits.size) for _ in range(world)]
            dist.all_gather(gathered, torch.from_numpy(st.logits.copy()))
            outs.append(np.concatenate([t.numpy() for t in gathered]))
        if rank == 0:
            results.put(np.stack(outs))
    finally:
        dist.destroy_process_group()


def test_shard_sizes_and_rejection():
    c = tiny_config()
    assert shard_sizes(c, 2) == {"heads": 4, "kv_heads": 1, "intermediate": 512, "vocab": 1024}
    with pytest.raises(ValueError):
        shard_sizes(c, 3)


def test_global_argmax_prefers_lowest_index_on_ties():
    assert global_argmax(np.array([1.0, 3.0, 3.0]), np.array([5, 900, 700])) == 700


def test_two_rank_sharded_oracle_equals_unsharded():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_oracle_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = results.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ck = synthetic_checkpoint(tiny_config(), seed=SEED)
    full = oracle_model(ck, attn_splits=2)
    st = full.new_state(32)
    want = np.stack([full.forward_token(int(t), st).copy() for t in synthetic_prompt(ck.config, STEPS, seed=SEED)])
    np.testing.assert_array_equal(got, want)


def _tp_gpu_rank(rank, world, port, config_name, results, graph=False, comm="p2p"):
    import datetime

    from harsh4b_b200.synthetic import qwen3_4b_config
    from harsh4b_b200.tp import TensorParallelQwen

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        config = tiny_config() if config_name == "tiny" else qwen3_4b_config(num_hidden_layers=2)
        ck = synthetic_checkpoint(config, seed=SEED)
        model = TensorParallelQwen(ck, kv_dtype="float16", attn_splits=16, comm=comm)
        prompt = synthetic_prompt(config, STEPS, seed=SEED)
        state = model.new_state(2 * STEPS)
        rows, greedy = [], []
        fed = list(prompt)
        for i in range(2 * STEPS):
            token, local = model.forward_token(int(fed[i]), state, graph=graph)
            parts = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(parts, local)
            rows.append(torch.cat(parts).cpu().numpy())
            if i >= STEPS - 1:
                greedy.append(token)
                if i + 1 < 2 * STEPS:
                    fed.append(token)
        torch.cuda.synchronize()
        model.close()
        if rank == 0:
            results.put((np.stack(rows), greedy, int(model.model.status())))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("config_name,graph,comm", [("tiny", False, "nccl"), ("qwen3_4b_2layer", True, "nccl"),
                                                    ("tiny", False, "p2p"), ("tiny", True, "p2p"),
                                                    ("qwen3_4b_2layer", False, "p2p"), ("qwen3_4b_2layer", True, "p2p")])
def test_two_gpu_tensor_parallel_matches_oracle(config_name, graph, comm):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from harsh4b_b200.synthetic import qwen3_4b_config

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_gpu_rank, args=(r, 2, port, config_name, results, graph, comm))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        rows, greedy, status = results.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    config = tiny_config() if config_name == "tiny" else qwen3_4b_config(num_hidden_layers=2)
    ck = synthetic_checkpoint(config, seed=SEED)
    reference = oracle_model(ck, kv_dtype=np.float16, attn_splits=16)
    st = reference.new_state(2 * STEPS)
    fed = list(synthetic_prompt(config, STEPS, seed=SEED))
    want, want_greedy = [], []
    for i in range(2 * STEPS):
        want.append(reference.forward_token(int(fed[i]), st).copy())
        if i >= STEPS - 1:
            want_greedy.append(int(np.argmax(want[-1])))
            if i + 1 < 2 * STEPS:
                fed.append(want_greedy[-1])
    np.testing.assert_array_equal(rows, np.stack(want))
    assert greedy == want_greedy
    assert status == 0


def _tp_prefill_rank(rank, world, port, results, attention="exact"):
    import datetime

    from harsh4b_b200.synthetic import qwen3_4b_config
    from harsh4b_b200.tp import TensorParallelQwen

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        config = qwen3_4b_config(num_hidden_layers=2)
        ck = synthetic_checkpoint(config, seed=SEED)
        model = TensorParallelQwen(ck, kv_dtype="float16", attn_splits=16, comm="nccl")
        prompt = synthetic_prompt(config, PREFILL, seed=SEED)
        state = model.new_state(PREFILL + STEPS)
        token, local = model.prefill(prompt, state, max_tokens=PREFILL_CHUNK, attention=attention)
        rows, greedy = [], [token]

        def gather(local):
            parts = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(parts, local)
            return torch.cat(parts).cpu().numpy()

        rows.append(gather(local))
        for _ in range(STEPS - 1):
            token, local = model.forward_token(greedy[-1], state)
            rows.append(gather(local))
            greedy.append(token)
        torch.cuda.synchronize()
        model.close()
        if rank == 0:
            results.put((np.stack(rows), greedy, int(model.model.status())))
    finally:
        dist.destroy_process_group()


PREFILL, PREFILL_CHUNK = 40, 24


@pytest.mark.gpu
def test_two_gpu_tensor_parallel_prefill_matches_oracle():
    """Sharded prefill (two chunks of prompt rows) then sharded decode, on
    two GPUs, against the unsharded oracle with the same attention splits
    (one per prompt query, 16 for decode): logits bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from harsh4b_b200.synthetic import qwen3_4b_config

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_prefill_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        rows, greedy, status = results.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    config = qwen3_4b_config(num_hidden_layers=2)
    ck = synthetic_checkpoint(config, seed=SEED)
    reference = oracle_model(ck, kv_dtype=np.float16, attn_splits=lambda ctx: 1 if ctx <= PREFILL else 16)
    st = reference.new_state(PREFILL + STEPS)
    for token in synthetic_prompt(config, PREFILL, seed=SEED):
        last = reference.forward_token(int(token), st).copy()
    want, want_greedy = [last], [int(np.argmax(last))]
    for _ in range(STEPS - 1):
        want.append(reference.forward_token(want_greedy[-1], st).copy())
        want_greedy.append(int(np.argmax(want[-1])))
    np.testing.assert_array_equal(rows, np.stack(want))
    assert greedy == want_greedy
    assert status == 0


@pytest.mark.gpu
def test_two_gpu_tensor_parallel_prefill_with_tensor_core_attention():
    """The sharded prefill with the tcgen05 prompt attention equals the
    single-GPU tcgen05 prefill bit for bit: each kv head's attention is the
    same kernel on the same rows, the attended rows are quantised with the
    global absmax and the o / down sums are exact int32 all-reduces; the
    decode after it is the oracle-exact one."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.synthetic import qwen3_4b_config

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_prefill_rank, args=(r, 2, port, results, "tensor")) for r in range(2)]
    for p in procs:
        p.start()
    try:
        rows, greedy, status = results.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert status == 0
    config = qwen3_4b_config(num_hidden_layers=2)
    ck = synthetic_checkpoint(config, seed=SEED)
    model = CudaQwen.from_checkpoint(ck, kv_dtype="float16", mode="chain", attn_splits=16)
    state = model.new_state(PREFILL + STEPS)
    prompt = synthetic_prompt(config, PREFILL, seed=SEED)
    want = [model.prefill(prompt, state, max_tokens=PREFILL_CHUNK, attention="tensor").cpu().numpy().copy()]
    want_greedy = [int(np.argmax(want[-1]))]
    for _ in range(STEPS - 1):
        want.append(model.forward_token(want_greedy[-1], state).cpu().numpy().copy())
        want_greedy.append(int(np.argmax(want[-1])))
    np.testing.assert_array_equal(rows, np.stack(want))
    assert greedy == want_greedy
    assert model.status() == 0
    state.close()
