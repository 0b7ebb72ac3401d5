"""The HTTP API server (laicompute_b200/bin/laic_server, laic::ApiServer; the reference's
routes of src/server_runtime.cpp:29-39) on the CPU: every route that needs no loaded model
(listing, status, upload, unload, stop, CORS preflight, the refusals without a model, 404s).
Generation through the server is covered by tests/test_gpu_server.py."""
import http.client
import json
import os
import socket
import subprocess
import tempfile
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SERVER = os.path.join(ROOT, "laicompute_b200", "bin", "laic_server")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Server:
    """laic_server on a free port over `model_dir`, stopped on exit (its own process only)."""

    def __init__(self, model_dir: str, cwd: str):
        self.port = free_port()
        self.proc = subprocess.Popen([SERVER, str(self.port), model_dir], cwd=cwd, stdout=subprocess.PIPE,
                                     stderr=subprocess.STDOUT)
        deadline = time.time() + 30
        while time.time() < deadline:
            try:
                socket.create_connection(("127.0.0.1", self.port), timeout=0.5).close()
                return
            except OSError:
                if self.proc.poll() is not None:
                    raise RuntimeError("laic_server exited: " + self.proc.stdout.read().decode(errors="replace"))
                time.sleep(0.05)
        raise RuntimeError("laic_server did not start listening")

    def request(self, method: str, path: str, body=None, headers=None, timeout: float = 60):
        c = http.client.HTTPConnection("127.0.0.1", self.port, timeout=timeout)
        data = body if isinstance(body, (bytes, type(None))) else json.dumps(body).encode()
        c.request(method, path, body=data, headers=headers or {})
        r = c.getresponse()
        raw = r.read()
        c.close()
        return r.status, dict(r.getheaders()), raw

    def json(self, method: str, path: str, body=None, headers=None):
        status, hdrs, raw = self.request(method, path, body, headers)
        return status, json.loads(raw) if raw else None

    def close(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@pytest.fixture(scope="module")
def server():
    if not os.path.exists(SERVER):
        pytest.skip("laic_server not built")
    with tempfile.TemporaryDirectory() as d:
        models = os.path.join(d, "models")
        with Server(models, cwd=d) as s:
            yield s


def test_status_and_empty_listing(server):
    assert server.json("GET", "/api/models") == (200, [])
    status, st = server.json("GET", "/api/status")
    assert status == 200
    assert st["generating"] is False and st["loaded"] == "" and st["tokens"] == 0
    assert st["cpu_logical"] >= 1 and st["cpu_physical"] >= 1 and 0 <= st["ram_percent"] <= 100


def test_generation_needs_a_model(server):
    for path in ("/api/chat", "/api/chat/stream"):
        status, body = server.json("POST", path, {"message": "hi", "max_tokens": 4})
        assert status == 409 and body == {"error": "no model loaded"}


def test_upload_list_and_refusals(server):
    status, body = server.json("POST", "/api/models/upload", b"not a gguf", {"X-Filename": "x.gguf"})
    assert status == 400
    status, body = server.json("POST", "/api/models/upload", b"GGUF" + bytes(60), {"X-Filename": "../m.bin"})
    assert status == 400  # not a .gguf name
    payload = b"GGUF" + bytes(range(256)) * 4
    status, body = server.json("POST", "/api/models/upload", payload, {"X-Filename": "sub/dir/tiny.gguf"})
    assert status == 201 and body == {"name": "tiny.gguf", "size": len(payload)}
    assert server.json("GET", "/api/models") == (200, [{"name": "tiny.gguf", "size": len(payload), "loaded": False}])
    status, body = server.json("POST", "/api/models/load", {"name": "missing.gguf"})
    assert status == 400 and body == {"error": "model not found"}


def test_stop_unload_preflight_and_unknown_routes(server):
    assert server.json("POST", "/api/stop") == (200, {"ok": True, "stopping": True})
    assert server.json("POST", "/api/models/unload") == (200, {"ok": True})
    status, hdrs, _ = server.request("OPTIONS", "/api/chat")
    assert status == 200 and hdrs.get("Access-Control-Allow-Origin") == "*"
    assert server.json("GET", "/api/nothing") == (404, {"error": "not found"})
    status, body = server.json("GET", "/")
    assert status == 404 and "index_v2.html" in body["error"]
