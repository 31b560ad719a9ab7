"""The reference chat server with the documented edits (tests/
reference_patches.py WEB_UI, applied to a temporary copy of web_ui.py):
for a runtime that declares ``concurrent = True`` (BatchedCudaBackend) two
requests stream at the same time instead of queueing on the model lock.
The runtime here is a CPU stand-in whose stream() only finishes when two
requests are inside it at once."""
import http.client
import importlib.util
import json
import sys
import threading

import pytest

from conftest import REFERENCE_ROOT, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="needs the reference checkout")


class _Tokenizer:
    def format(self, system, messages, budget):
        return " ".join(m["content"] for m in messages)

    def encode(self, text):
        return [len(word) for word in text.split()]


class _ConcurrentRuntime:
    concurrent = True
    max_context = 2048
    device, hardware, description = "cuda", "stand-in", "stand-in"

    def __init__(self):
        self.tokenizer = _Tokenizer()
        self.both_inside = threading.Barrier(2, timeout=20)

    def status(self):
        return {"runtime": self.device, "ready": True}

    def stream(self, ids, max_tokens, temperature, cancelled):
        self.both_inside.wait()  # raises BrokenBarrierError if the requests were serialised
        yield {"token": "ok", "done": False}
        yield {"done": True, "stats": {"tokens": 1}}


def _post(port, request_id, out):
    connection = http.client.HTTPConnection("127.0.0.1", port, timeout=60)
    body = json.dumps({"request_id": request_id, "messages": [{"role": "user", "content": "hello there"}],
                       "max_tokens": 4, "temperature": 0})
    connection.request("POST", "/api/chat", body, {"Content-Type": "application/json"})
    out[request_id] = connection.getresponse().read().decode()


def test_web_ui_streams_concurrent_requests_for_a_concurrent_runtime(tmp_path):
    from reference_patches import WEB_UI, apply

    patched = tmp_path / "web_ui_cuda.py"
    patched.write_text(apply((REFERENCE_ROOT / "web_ui.py").read_text(), WEB_UI))
    sys.path.insert(0, str(REFERENCE_ROOT))
    try:
        spec = importlib.util.spec_from_file_location("web_ui_cuda", patched)
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
    finally:
        sys.path.remove(str(REFERENCE_ROOT))
    server = module.InferenceServer(("127.0.0.1", 0), _ConcurrentRuntime())
    thread = threading.Thread(target=server.serve_forever, daemon=True)
    thread.start()
    try:
        out = {}
        clients = [threading.Thread(target=_post, args=(server.server_port, f"req{i}", out)) for i in range(2)]
        for c in clients:
            c.start()
        for c in clients:
            c.join(timeout=60)
    finally:
        server.shutdown()
        server.server_close()
    for i in range(2):
        assert '"token": "ok"' in out[f"req{i}"] and '"error"' not in out[f"req{i}"]
