"""Benchmark-suite integration: the reference's own measurement core
(benchmarks/bench_energy.py timed_generate, reused by bench_latency.py)
driving the backend composed with its Runtime (CPU, oracle model handed in),
and harsh4b_b200.benchsuite's grid and energy measurement on the GPU."""
import sys
import types

import numpy as np
import pytest

from conftest import REFERENCE_ROOT, reference_available

pytest.importorskip("tokenizers")


@pytest.mark.skipif(not reference_available(), reason="needs the reference checkout")
def test_reference_timed_generate_drives_the_backend():
    from test_runtime import _OracleModel, _Tokenizer, _tiny

    from harsh4b_b200 import benchsuite
    from harsh4b_b200.runtime import CudaBackend

    for path in (REFERENCE_ROOT, REFERENCE_ROOT / "benchmarks"):
        sys.path.insert(0, str(path))
    try:
        import bench_energy
        import inference_runtime
    finally:
        for path in (REFERENCE_ROOT, REFERENCE_ROOT / "benchmarks"):
            sys.path.remove(str(path))

    class CudaRuntime(CudaBackend, inference_runtime.Runtime):
        pass

    checkpoint, prompt = _tiny()
    greedy = lambda logits, generated, temperature: int(np.argmax(logits))  # noqa: E731
    runtime = CudaRuntime(model=_OracleModel(checkpoint), tokenizer=_Tokenizer(2048, stop_ids=()), sampler=greedy)
    # sync_logits calls runtime.torch.cuda.synchronize() for "cuda": no device here
    runtime.torch = types.SimpleNamespace(cuda=types.SimpleNamespace(synchronize=lambda *a: None))
    theirs = bench_energy.timed_generate(runtime, prompt, 6, 0.0)
    ours = benchsuite.timed_generate(runtime, prompt, 6, 0.0)
    assert theirs["generated"] == ours["generated"] and len(theirs["generated"]) == 6
    assert len(theirs["itls"]) == len(ours["itls"]) == 5
    assert theirs["ttft"] > 0 and theirs["decode_s"] > 0


def test_percentile_matches_linear_interpolation():
    from harsh4b_b200.benchsuite import percentile

    assert percentile([], 95) == 0.0
    assert percentile([3.0, 1.0, 2.0], 50) == 2.0
    assert abs(percentile([1.0, 2.0, 3.0, 4.0], 95) - 3.85) < 1e-12


@pytest.mark.gpu
def test_latency_grid_and_energy_on_the_gpu():
    from test_runtime import _Tokenizer

    from harsh4b_b200 import benchsuite
    from harsh4b_b200.model import CudaQwen
    from harsh4b_b200.runtime import CudaBackend
    from harsh4b_b200.synthetic import synthetic_checkpoint, tiny_config

    model = CudaQwen.from_checkpoint(synthetic_checkpoint(tiny_config(), seed=3))
    backend = CudaBackend(model=model, tokenizer=_Tokenizer(model.vocab, stop_ids=()))
    cells = benchsuite.latency_grid(backend, [8, 16], [4], repeats=2, warmup=1, out=lambda *a: None)
    assert [(c["prompt_tokens"], c["decode_tokens"], c["generated_tokens"]) for c in cells] == [(8, 4, 4), (16, 4, 4)]
    for cell in cells:
        assert cell["ttft_med_s"] > 0 and cell["tpot_med_ms"] > 0 and cell["decode_med_tok_s"] > 0
    energy = benchsuite.energy_per_token(backend, list(range(32)), 16)
    assert energy["tokens"] == 16 and energy["joules"] >= 0 and energy["mean_watts"] > 0
