"""The edits a maintainer makes to the reference to route its "cuda" runtime
to this backend, as (file, old text, new text) replacements. INTEGRATION.md
shows the same edits as diffs; tests apply them to temporary copies of the
reference's files to check that they apply and work."""

INFERENCE_RUNTIME = [
    ('def create_runtime(name="auto", model_path=None, tokenizer_path=None, **options):',
     'from harsh4b_b200.runtime import CudaBackend\n'
     'from harsh4b_b200.serving import BatchedCudaBackend\n\n\n'
     'class CudaRuntime(CudaBackend, Runtime):\n'
     '    """B200 packed-int4 decode (harsh4b_b200)."""\n\n\n'
     'class BatchedCudaRuntime(BatchedCudaBackend, Runtime):\n'
     '    """B200 decode with concurrent requests batched (harsh4b_b200)."""\n\n\n'
     'def create_runtime(name="auto", model_path=None, tokenizer_path=None, **options):'),
    ('cls = MLXRuntime if selected == "mlx" else LiteSparkRuntime if selected == "cpu" else TorchRuntime',
     'cls = MLXRuntime if selected == "mlx" else LiteSparkRuntime if selected == "cpu" else (\n'
     '        BatchedCudaRuntime if options.get("slots", 1) > 1 else CudaRuntime)'),
]

WEB_UI = [
    ('import argparse\n', 'import argparse\nimport contextlib\n'),
    ('            with self.server.model_lock:\n'
     '                for payload in runtime.stream(ids, max_tokens, temperature, cancelled):',
     '            serial = contextlib.nullcontext() if getattr(runtime, "concurrent", False) else self.server.model_lock\n'
     '            with serial:\n'
     '                for payload in runtime.stream(ids, max_tokens, temperature, cancelled):'),
    ('    parser.add_argument("--port", type=int, default=7860)\n',
     '    parser.add_argument("--port", type=int, default=7860)\n'
     '    parser.add_argument("--batch-slots", type=int, default=1,\n'
     '                        help="cuda: batch up to this many concurrent requests")\n'),
    ('        args.runtime, args.model, args.tokenizer, cpu_threads=args.cpu_threads\n    )',
     '        args.runtime, args.model, args.tokenizer, cpu_threads=args.cpu_threads,\n'
     '        **({"slots": args.batch_slots} if args.batch_slots > 1 else {})\n    )'),
]

TEST_PY = [
    ('parser.add_argument("--runtime", choices=("mlx", "cpu"), default="cpu",',
     'parser.add_argument("--runtime", choices=("mlx", "cpu", "cuda"), default="cpu",'),
    ('    if args.runtime == "cpu":\n        run_cpu(args, tokens, tokenizer)\n        return\n',
     '    if args.runtime == "cpu":\n        run_cpu(args, tokens, tokenizer)\n        return\n'
     '    if args.runtime == "cuda":\n'
     '        from harsh4b_b200.cli import run_test_py\n'
     '        run_test_py(args, tokens, tokenizer, MODEL_PATH)\n'
     '        return\n'),
]


def apply(text: str, patches) -> str:
    for old, new in patches:
        if text.count(old) != 1:
            raise ValueError(f"patch anchor not found exactly once: {old[:60]!r}")
        text = text.replace(old, new)
    return text
