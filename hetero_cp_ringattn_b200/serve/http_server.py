"""OpenAI-style HTTP API: POST /v1/completions (+ SSE streaming), GET /health, GET /metrics.

Parity: rust/src/api/server.rs:39-205 and api/types.rs:4-142: request fields (`model`, `prompt`,
`max_tokens` default 20, `temperature` 0.0, `top_p` 1.0, `stream`, `stop`, `session_id`,
`keep_kv`, `append`), fail-closed session validation (append / keep_kv require session_id ->
400), `text_completion` responses with usage, SSE chunks terminated by `data: [DONE]`,
`/health` {status, workers_connected, num_domains} and `/metrics` {total, completed, failed,
queued, active}. Served by the standard library's threaded HTTP server (no extra dependency).
"""

from __future__ import annotations

import json
import queue
import select
import socket
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Optional

from ..errors import Overloaded, ProtocolError
from .scheduler import Job


def validate_session_fields(body: dict) -> Optional[str]:
    if body.get("append") and not body.get("session_id"):
        return "append=true requires session_id"
    if body.get("keep_kv") and not body.get("session_id"):
        return "keep_kv=true requires session_id"
    return None


MAX_BODY_BYTES = 64 << 20   # a 1M-token prompt as text is a few MB

# request fields and the JSON types they accept (the reference's CompletionRequest, api/types.rs:
# a value of the wrong type is a 422 there too)
_FIELD_TYPES = {"model": (str,), "max_tokens": (int,), "temperature": (int, float),
                "top_p": (int, float), "stream": (bool,), "session_id": (str,), "keep_kv": (bool,),
                "append": (bool,), "ignore_eos": (bool,)}


def _field_type_error(body: dict) -> Optional[str]:
    for name, types in _FIELD_TYPES.items():
        v = body.get(name)
        if v is None:
            continue
        if not isinstance(v, types) or (bool not in types and isinstance(v, bool)):
            return f"{name}: expected {' or '.join(t.__name__ for t in types)}"
    if "max_tokens" in body and body["max_tokens"] is not None and body["max_tokens"] < 1:
        return "max_tokens: must be at least 1"
    if body.get("temperature") is not None and body["temperature"] < 0:
        return "temperature: must not be negative"
    if body.get("top_p") is not None and not 0 < body["top_p"] <= 1:
        return "top_p: must be in (0, 1]"
    stop = body.get("stop")
    if stop is not None and not (isinstance(stop, str) or
                                 (isinstance(stop, list) and all(isinstance(x, str) for x in stop))):
        return "stop: expected a string or a list of strings"
    return None


def _peer_closed(sock) -> bool:
    """True once the client has closed its end of the connection: the socket polls readable
    (or hung up) and a non-blocking peek returns no bytes. A request pipelined behind this one
    peeks as data, not a close. poll() has no descriptor-number limit (select() fails for
    descriptors >= FD_SETSIZE, which a busy server reaches), and only an orderly shutdown or a
    reset counts as closed."""
    try:
        poller = select.poll()
        poller.register(sock, select.POLLIN | select.POLLHUP | select.POLLERR)
        if not poller.poll(0):
            return False
    except ValueError:            # the socket was already closed on this side (fileno -1)
        return True
    try:
        return sock.recv(1, socket.MSG_PEEK | socket.MSG_DONTWAIT) == b""
    except (BlockingIOError, InterruptedError):
        return False
    except (ConnectionResetError, BrokenPipeError, ConnectionAbortedError):
        return True
    except OSError:
        return False


class _WindowDeltas:
    """Incremental detokenization over a sliding window: decode the tokens since `prefix`
    (already streamed, kept as left context so merges and leading spaces decode as in the full
    text) and return what the tokens from `read` on add. A trailing partial character (a
    multi-byte character split over tokens decodes to U+FFFD until its last byte arrives) is held
    back until it completes or the stream ends. Linear in the stream length."""

    def __init__(self, tok):
        self.tok, self.ids, self.prefix, self.read = tok, [], 0, 0

    def __call__(self, token: int, last: bool) -> str:
        self.ids.append(token)
        done = self.tok.decode(self.ids[self.prefix:self.read]) if self.read > self.prefix else ""
        text = self.tok.decode(self.ids[self.prefix:])
        if not last and (text.endswith("\ufffd") or len(text) <= len(done)):
            return ""
        self.prefix, self.read = self.read, len(self.ids)
        return text[len(done):]


class _StopStringDeltas:
    """Deltas for a request with stop strings: the whole text is decoded each token and the
    last (longest stop - 1) characters are held back until they cannot start a stop string, so
    no part of a stop sequence is ever streamed (cost grows with the generation length; only
    requests that set `stop` pay it)."""

    def __init__(self, tok, stops):
        self.tok, self.stops, self.ids, self.sent = tok, stops, [], 0
        self.hold = max(len(x) for x in stops) - 1

    def __call__(self, token: int, last: bool) -> str:
        self.ids.append(token)
        text = _cut_at_stop(self.tok.decode(self.ids), self.stops)
        upto = len(text)
        if not last:
            upto -= self.hold
            if text.endswith("\ufffd"):
                upto = min(upto, len(text) - 1)
        delta = text[self.sent:max(self.sent, upto)]
        self.sent = max(self.sent, upto)
        return delta


def _cut_at_stop(text: str, stops) -> str:
    """The text before the earliest stop string (OpenAI semantics: the stop is not returned)."""
    if not stops:
        return text
    cut = min((i for i in (text.find(x) for x in stops if x) if i >= 0), default=-1)
    return text if cut < 0 else text[:cut]


class ApiState:
    def __init__(self, coordinator, tokenizer, model_name: str, num_domains: int,
                 vocab_size: Optional[int] = None):
        self.coord = coordinator
        self.tok = tokenizer
        cfg = getattr(coordinator, "cfg", None)
        self.vocab_size = vocab_size or getattr(cfg, "vocab_size", None) or \
            getattr(tokenizer, "vocab_size", None) or (1 << 31)
        self.model_name = model_name
        self.num_domains = num_domains
        self.workers_connected = num_domains


def make_handler(state: ApiState):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, fmt, *args):  # quiet
            pass

        def _json(self, code: int, obj) -> None:
            data = json.dumps(obj).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.send_header("Access-Control-Allow-Origin", "*")
            self.end_headers()
            self.wfile.write(data)

        def _text(self, code: int, msg: str) -> None:
            data = msg.encode()
            self.send_response(code)
            self.send_header("Content-Type", "text/plain; charset=utf-8")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path == "/health":
                failed = getattr(state.coord, "control_failed", None)
                if failed:   # a rank is gone: the job must be restarted (no elastic recovery)
                    return self._json(503, {"status": "unhealthy", "workers_connected": 0,
                                            "num_domains": state.num_domains, "error": failed})
                return self._json(200, {"status": "ok", "workers_connected": state.workers_connected,
                                        "num_domains": state.num_domains})
            if self.path == "/v1/models":   # for OpenAI-style clients and benchmark tools
                return self._json(200, {"object": "list", "data": [
                    {"id": state.model_name, "object": "model", "owned_by": "hcp-b200"}]})
            if self.path == "/metrics/prometheus":
                data = state.coord.metrics.prometheus(state.coord.sched.queued,
                                                      len(state.coord.sched.active)).encode()
                self.send_response(200)
                self.send_header("Content-Type", "text/plain; version=0.0.4; charset=utf-8")
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)
                return None
            if self.path == "/metrics":
                m = state.coord.metrics
                return self._json(200, {"total_requests": m.total, "completed_requests": m.completed,
                                        "failed_requests": m.failed,
                                        "queued_requests": state.coord.sched.queued,
                                        "active_requests": len(state.coord.sched.active)})
            return self._text(404, "not found")

        def do_POST(self):
            if self.path != "/v1/completions":
                return self._text(404, "not found")
            try:
                n = int(self.headers.get("Content-Length", "0"))
            except ValueError:
                return self._text(400, "bad Content-Length")
            if n < 0 or n > MAX_BODY_BYTES:
                return self._text(413, f"request body over {MAX_BODY_BYTES} bytes")
            try:
                body = json.loads(self.rfile.read(n) or b"{}")
            except json.JSONDecodeError as e:
                return self._text(400, f"invalid JSON: {e}")
            prompt = body.get("prompt") if isinstance(body, dict) else None
            token_prompt = isinstance(prompt, list) and bool(prompt) and all(
                isinstance(t, int) and not isinstance(t, bool) for t in prompt)
            if not (isinstance(prompt, str) or token_prompt):
                return self._text(422, "prompt (a string or a list of token ids) is required")
            if token_prompt and not all(0 <= t < state.vocab_size for t in prompt):
                return self._text(422, f"prompt token ids must be in [0, {state.vocab_size})")
            bad = _field_type_error(body)
            if bad:
                return self._text(422, bad)
            err = validate_session_fields(body)
            coord = state.coord
            if err:
                coord.metrics.bump("total")
                coord.metrics.bump("failed")
                return self._text(400, err)
            rid = coord.next_request_id()
            created = int(time.time())
            model = body.get("model") or state.model_name
            ids = list(prompt) if token_prompt else state.tok.encode(prompt)
            stop = body.get("stop")
            stop_strings = [stop] if isinstance(stop, str) else [x for x in (stop or []) if x]
            events: "queue.Queue" = queue.Queue()
            job = Job(request_id=rid, prompt_ids=ids, max_tokens=int(body.get("max_tokens", 20)),
                      temperature=float(body.get("temperature", 0.0)),
                      top_p=float(body.get("top_p", 1.0)), session_id=body.get("session_id"),
                      keep_kv=bool(body.get("keep_kv", False)), append=bool(body.get("append", False)),
                      stop_strings=stop_strings or None,
                      ignore_eos=bool(body.get("ignore_eos", False)),
                      on_token=lambda t, fr: events.put(("tok", t, fr)),
                      done=lambda r: events.put(("done", r, None)))
            try:
                coord.submit(job)
            except Overloaded as e:
                return self._text(503, str(e))
            except ProtocolError as e:
                coord.metrics.bump("failed")
                return self._text(400, str(e))
            if body.get("stream"):
                return self._stream(rid, created, model, events, job, stop_strings)
            next_poll = 0.0
            while True:
                try:
                    kind, res, _ = events.get(timeout=0.05)
                except queue.Empty:
                    kind = None
                if kind == "done":
                    break
                now = time.monotonic()
                if now >= next_poll and not job.cancelled:
                    next_poll = now + 0.05
                    if _peer_closed(self.connection):
                        job.cancelled = True    # the client went away: stop generating for it
            if job.cancelled:
                return None                     # nobody is left to answer
            if "error" in res:
                return self._text(int(res.get("status", 500)), res["error"])
            text = _cut_at_stop(state.tok.decode(res["tokens"]), stop_strings)
            pt, ct = res["prompt_tokens"], len(res["tokens"])
            return self._json(200, {
                "id": f"hcp-completion-{rid}", "object": "text_completion", "created": created,
                "model": model,
                "choices": [{"text": text, "index": 0, "logprobs": None,
                             "finish_reason": res["finish_reason"]}],
                "usage": {"prompt_tokens": pt, "completion_tokens": ct, "total_tokens": pt + ct}})

        def _stream(self, rid, created, model, events, job, stops=None):
            """Server-sent events: one chunk per generated token, then `[DONE]`. A client that
            goes away cancels the job (the coordinator stops generating for it)."""
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()

            def send(data: str):
                try:
                    self.wfile.write(f"data: {data}\n\n".encode())
                    self.wfile.flush()
                except OSError:   # the client closed the stream: stop generating for it
                    job.cancelled = True
                    raise

            delta_of = _StopStringDeltas(state.tok, stops) if stops else _WindowDeltas(state.tok)
            while True:
                try:
                    kind, a, b = events.get(timeout=0.05)
                except queue.Empty:
                    # queued or still prefilling: no write fails yet, so look at the socket
                    if not job.cancelled and _peer_closed(self.connection):
                        job.cancelled = True
                    continue
                if kind == "tok":
                    chunk = {"id": f"hcp-completion-{rid}", "object": "text_completion",
                             "created": created, "model": model,
                             "choices": [{"text": delta_of(a, b is not None), "index": 0,
                                          "finish_reason": b}]}
                    send(json.dumps(chunk))
                elif kind == "done":
                    if "error" in a:
                        send(json.dumps({"error": a["error"]}))
                    break
            send("[DONE]")
            self.close_connection = True

        def handle_one_request(self):
            try:
                super().handle_one_request()
            except (BrokenPipeError, ConnectionResetError):
                self.close_connection = True   # client gone mid-stream; the job was cancelled

    return Handler


class ApiServer:
    def __init__(self, state: ApiState, host: str = "127.0.0.1", port: int = 0):
        self.httpd = ThreadingHTTPServer((host, port), make_handler(state))
        self.httpd.daemon_threads = True
        self.thread = None

    @property
    def port(self) -> int:
        return self.httpd.server_address[1]

    def start(self) -> "ApiServer":
        self.thread = threading.Thread(target=self.httpd.serve_forever, daemon=True)
        self.thread.start()
        return self

    def stop(self) -> None:
        self.httpd.shutdown()
        self.httpd.server_close()
