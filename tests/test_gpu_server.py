"""Generation through the HTTP API server (laic::ApiServer over LlamaRuntime; the reference's
routes of src/server_runtime.cpp:29-39) on the GPU: load a model, /api/chat and the
/api/chat/stream server-sent events give the text of the command-line generator (the same
greedy LlamaRuntime::generate_ids), /api/status follows the generation, /api/stop ends a
running stream through LlamaRuntime::request_stop, unload frees the model."""
import http.client
import json
import os
import shutil
import subprocess
import tempfile
import threading

import pytest

from test_server import Server, SERVER

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
GENERATE = os.path.join(ROOT, "laicompute_b200", "bin", "laic_generate")
MODEL = os.path.join(HERE, "golden", "tiny_q4.gguf")


def sse_events(port: int, body: dict, on_event=None, timeout: float = 120):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=timeout)
    c.request("POST", "/api/chat/stream", body=json.dumps(body).encode())
    r = c.getresponse()
    assert r.status == 200 and r.getheader("Content-Type") == "text/event-stream"
    events, buf = [], b""
    while True:
        chunk = r.read1(65536)
        if not chunk:
            break
        buf += chunk
        while b"\n\n" in buf:
            line, buf = buf.split(b"\n\n", 1)
            assert line.startswith(b"data: ")
            ev = json.loads(line[6:])
            events.append(ev)
            if on_event:
                on_event(ev)
    c.close()
    return events


@pytest.fixture(scope="module")
def loaded():
    with tempfile.TemporaryDirectory() as d:
        models = os.path.join(d, "models")
        os.makedirs(models)
        shutil.copy(MODEL, os.path.join(models, "tiny_q4.gguf"))
        with Server(models, cwd=d) as s:
            assert s.json("POST", "/api/models/load", {"name": "tiny_q4.gguf"}) == (200, {"ok": True})
            yield s


def test_chat_matches_the_command_line_generator(loaded):
    prompt, n = "Hello there", 12
    expect = subprocess.run([GENERATE, MODEL, prompt, str(n)], capture_output=True, text=True, check=True).stdout
    expect = expect[:-1] if expect.endswith("\n") else expect
    status, body = loaded.json("POST", "/api/chat", {"message": prompt, "max_tokens": n})
    assert status == 200 and body["stopped"] is False
    assert body["text"] == expect
    assert 1 <= body["tokens"] <= n and body["tokens_per_sec"] > 0
    events = sse_events(loaded.port, {"message": prompt, "max_tokens": n})
    assert events[-1]["done"] is True and events[-1]["stopped"] is False
    assert "".join(e["token"] for e in events[:-1]) == expect
    assert [e["tokens"] for e in events[:-1]] == list(range(1, len(events)))
    status, st = loaded.json("GET", "/api/status")
    assert st["generating"] is False and st["loaded"] == "tiny_q4.gguf" and st["tokens"] == len(events) - 1
    assert loaded.json("GET", "/api/models")[1][0]["loaded"] is True


def test_stop_ends_a_running_stream(loaded):
    stop_sent = threading.Event()

    def on_event(ev):
        if not stop_sent.is_set() and "token" in ev:
            stop_sent.set()
            assert loaded.json("POST", "/api/stop") == (200, {"ok": True, "stopping": True})

    events = sse_events(loaded.port, {"message": "Count with me", "max_tokens": 200}, on_event)
    done = events[-1]
    assert done["done"] is True and stop_sent.is_set()
    if done["stopped"]:  # the stop arrived before the 200th token (the usual case)
        assert done["tokens"] < 200
    # the next generation starts with the stop flag cleared
    status, body = loaded.json("POST", "/api/chat", {"message": "Hello there", "max_tokens": 3})
    assert status == 200 and body["stopped"] is False


def test_second_generation_is_refused_while_one_runs(loaded):
    started, result = threading.Event(), {}

    def on_event(ev):
        if not started.is_set():
            started.set()
            result["second"] = loaded.json("POST", "/api/chat", {"message": "x", "max_tokens": 2})
            result["status"] = loaded.json("GET", "/api/status")[1]

    events = sse_events(loaded.port, {"message": "Count with me", "max_tokens": 200}, on_event)
    if result["status"]["generating"]:  # (the usual case: the first stream was still running)
        assert result["second"] == (409, {"error": "generation already running"})
    assert events[-1]["done"] is True
