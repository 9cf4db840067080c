"""Private-network LoRA rollout RPC: authenticated JSON plus raw tensor packets, never pickle.

Wire protocol of the reference service (``rollout_manager/backends/vllm_lora_remote.py:96-346``),
so a learner here can drive that vLLM service and the native service below alike:

* one TCP connection per call; every JSON message is framed by a 4-byte big-endian length
  (32 MiB budget) and must contain only finite numbers;
* the client first sends ``{"token": ...}`` (32..256 chars of [A-Za-z0-9_-]); the server answers
  ``{"authenticated": true|false}`` (constant-time comparison);
* then ``{"operation": ..., "arguments": {...}}`` with operation in initialize / status /
  activate / sample_group / pause / resume / close; ``activate`` is followed by one LoRA
  update frame (``lora_transport``), read only after authentication;
* the reply is ``{"ok": true, "result": ...}`` or ``{"ok": false, "error": ..., ...}``.

Endpoints must be private or loopback IPv4. A client that saw any failure refuses everything but
status/close (an unknown outcome is never retried); the server latches failure likewise.
``sample_group`` takes 1..32 specs ``{prompt_ids, max_tokens, temperature, request_id (32 hex),
sampling_seed}``.
"""

from __future__ import annotations

import asyncio
import copy
import hmac
import ipaddress
import json
import math
import re
import socket
import socketserver
import struct
import sys
import threading

from ..rl.lora_config import DistributedLoRAConfig
from .lora_transport import _read_exact, receive_update, send_update

MAX_JSON_BYTES = 32 << 20
_SPEC_FIELDS = {"prompt_ids", "max_tokens", "temperature", "request_id", "sampling_seed"}
OPERATIONS = {"initialize", "status", "activate", "sample_group", "pause", "resume", "close"}
_PRIVATE = tuple(ipaddress.ip_network(n) for n in ("10.0.0.0/8", "172.16.0.0/12", "192.168.0.0/16", "127.0.0.0/8"))


def check_endpoint(address) -> tuple[str, int]:
    host, port = address
    ip = ipaddress.IPv4Address(host)
    if not any(ip in net for net in _PRIVATE) or type(port) is not int or not 0 <= port <= 65535:
        raise ValueError("RPC requires an explicit private or loopback IPv4 address and valid port")
    return str(ip), port


def check_token(value) -> str:
    if not isinstance(value, str) or not re.fullmatch(r"[A-Za-z0-9_-]{32,256}", value):
        raise ValueError("RPC token requires 32..256 ASCII letters, digits, underscores or hyphens")
    return value


def send_json(stream, value) -> None:
    data = json.dumps(value, separators=(",", ":"), allow_nan=False).encode()
    if not 0 < len(data) <= MAX_JSON_BYTES:
        raise ValueError("RPC JSON exceeds byte budget")
    stream.sendall(struct.pack("!I", len(data)) + data)


def receive_json(stream, limit: int = MAX_JSON_BYTES):
    (size,) = struct.unpack("!I", _read_exact(stream, 4))
    if not 0 < size <= limit:
        raise ValueError("RPC JSON exceeds byte budget")

    def reject(_):
        raise ValueError("RPC JSON requires finite values")

    return json.loads(_read_exact(stream, size), parse_constant=reject)


def check_specs(values):
    if not isinstance(values, list) or not 1 <= len(values) <= 32:
        raise ValueError("sample_group requires 1..32 request specifications")
    seen = set()
    for spec in values:
        if not isinstance(spec, dict) or set(spec) != _SPEC_FIELDS:
            raise ValueError("invalid sample request fields")
        ids, rid = spec["prompt_ids"], spec["request_id"]
        ok = (isinstance(ids, list) and 1 <= len(ids) <= 4096 and all(type(t) is int and 0 <= t < 2 ** 31 for t in ids)
              and type(spec["max_tokens"]) is int and 1 <= spec["max_tokens"] <= 4096
              and type(spec["temperature"]) in (int, float) and math.isfinite(spec["temperature"])
              and 0 < spec["temperature"] <= 10 and isinstance(rid, str) and re.fullmatch(r"[0-9a-f]{32}", rid)
              and rid not in seen and type(spec["sampling_seed"]) is int and 0 <= spec["sampling_seed"] < 2 ** 63 - 1)
        if not ok:
            raise ValueError("invalid bounded sample request or duplicate request ID")
        seen.add(rid)
    return values


class RemoteLoRAClient:
    """Synchronous client; the first error latches failure (only status/close stay allowed)."""

    def __init__(self, host, port, token, *, timeout: float = 7200) -> None:
        self.address, self._token = check_endpoint((host, port)), check_token(token)
        if type(timeout) not in (int, float) or not math.isfinite(timeout) or not 0 < timeout <= 7200:
            raise ValueError("RPC timeout must be finite and at most 7200 seconds")
        self.timeout, self.failed, self.closed = timeout, False, False
        self._lock = threading.Lock()
        self.ack = self.activation_receipts = self.base_identity = None

    def _call(self, operation, arguments=None, update=None):
        if operation not in OPERATIONS:
            raise ValueError("unknown RPC operation")
        with self._lock:
            if self.closed or (self.failed and operation not in {"status", "close"}):
                raise RuntimeError("remote client has a closed or unknown prior outcome; no retry is allowed")
            try:
                with socket.create_connection(self.address, timeout=self.timeout) as stream:
                    send_json(stream, {"token": self._token})
                    if receive_json(stream, 4096) != {"authenticated": True}:
                        raise PermissionError("remote authentication rejected")
                    send_json(stream, {"operation": operation, "arguments": arguments or {}})
                    if update is not None:
                        send_update(stream, *update)
                    response = receive_json(stream)
                if not isinstance(response, dict) or response.get("ok") is not True or "result" not in response:
                    detail = (f"{response.get('error_type', 'UnknownError')}: {response.get('reason', 'outcome unknown')}"
                              if isinstance(response, dict) else "invalid response; outcome unknown")
                    raise RuntimeError(f"remote {operation} failed: {detail}")
                return response["result"]
            except BaseException:
                self.failed = True
                raise

    def initialize(self, *, lora_config=None):
        profile = DistributedLoRAConfig() if lora_config is None else DistributedLoRAConfig.from_dict(lora_config)
        result = self._call("initialize", {"lora_config": profile.to_dict()})
        try:
            if DistributedLoRAConfig.from_dict(result["lora_config"]) != profile:
                raise ValueError("rollout LoRA configuration differs from the learner profile")
            self.base_identity = result["base_identity"]
        except (KeyError, TypeError, ValueError) as error:
            self.failed = True
            raise RuntimeError("remote initialize returned an invalid LoRA configuration") from error
        return result

    def status(self):
        return self._call("status")

    def activate(self, manifest, payload):
        result = self._call("activate", update=(manifest, payload))
        self.ack, self.activation_receipts = result["ack"], result["activation_receipts"]
        return result

    def sample_group(self, specs):
        return self._call("sample_group", {"specs": check_specs(specs)})

    def pause(self):
        return self._call("pause")

    def resume(self):
        return self._call("resume")

    def close(self):
        if self.closed:
            return {"closed": True, "drain_complete": True}
        result = self._call("close")
        self.closed = True
        return result


class _Handler(socketserver.BaseRequestHandler):
    def handle(self):
        authenticated, operation = False, "authentication"
        server = self.server
        try:
            self.request.settimeout(5)
            auth = receive_json(self.request, 4096)
            if (not isinstance(auth, dict) or set(auth) != {"token"} or not isinstance(auth["token"], str)
                    or not hmac.compare_digest(auth["token"].encode(), server.token.encode())):
                send_json(self.request, {"authenticated": False})
                return
            send_json(self.request, {"authenticated": True})
            authenticated = True
            self.request.settimeout(server.io_timeout)
            req = receive_json(self.request)
            if (not isinstance(req, dict) or set(req) != {"operation", "arguments"} or req["operation"] not in OPERATIONS
                    or not isinstance(req["arguments"], dict)):
                raise ValueError("invalid RPC request envelope")
            operation = req["operation"]
            update = receive_update(self.request) if operation == "activate" else None
            future = asyncio.run_coroutine_threadsafe(server.dispatch(operation, req["arguments"], update), server.loop)
            send_json(self.request, {"ok": True, "result": future.result(timeout=server.io_timeout)})
        except Exception as error:
            response = {"ok": False, "error": "remote operation rejected or outcome unknown"}
            if authenticated:
                server.failed = True
                reason = (str(error) or "RPC timeout or unknown outcome").replace(server.token, "<redacted>")[:2048]
                response.update(error_type=type(error).__name__, reason=reason)
                print(f"LoRA RPC {operation}: {type(error).__name__}: {reason}", file=sys.stderr, flush=True)
            try:
                send_json(self.request, response)
            except OSError:
                pass


class RemoteLoRAServer(socketserver.ThreadingTCPServer):
    """Serves one rollout controller (the vLLM actor, or ``NativeRolloutController``).

    The controller provides ``start()``, ``activate(manifest, payload) -> ack``,
    ``sample_batch(specs) -> results``, ``pause()``, ``resume()``, ``close()`` (coroutines except
    ``sample_batch``), and ``state``, ``ack``, ``base_identity``, ``lora_config``,
    ``activation_receipts``."""

    daemon_threads = True
    request_queue_size = 8

    def __init__(self, address, token, controller, *, io_timeout: float = 7200) -> None:
        address, self.token = check_endpoint(address), check_token(token)
        if type(io_timeout) not in (int, float) or not math.isfinite(io_timeout) or not 0 < io_timeout <= 7200:
            raise ValueError("server RPC timeout must be finite and at most 7200 seconds")
        self.controller, self.io_timeout, self.failed = controller, io_timeout, False
        self._slots, self._busy = threading.BoundedSemaphore(8), False
        super().__init__(address, _Handler)
        self.loop = asyncio.new_event_loop()
        self._thread = threading.Thread(target=self.loop.run_forever, daemon=True)
        self._thread.start()

    def process_request(self, request, client_address):
        if not self._slots.acquire(blocking=False):
            self.shutdown_request(request)
            return
        try:
            super().process_request(request, client_address)
        except BaseException:
            self._slots.release()
            raise

    def process_request_thread(self, request, client_address):
        try:
            super().process_request_thread(request, client_address)
        finally:
            self._slots.release()

    def _status(self) -> dict:
        c = self.controller
        return {"state": c.state, "failed": self.failed or c.state == "failed", "policy_ack": copy.deepcopy(c.ack),
                "base_identity": copy.deepcopy(c.base_identity), "lora_config": c.lora_config.to_dict(),
                "activation_receipts": copy.deepcopy(c.activation_receipts)}

    async def dispatch(self, operation, arguments, update):
        c = self.controller
        if operation == "status" and not arguments:
            return self._status()
        if operation == "close" and not arguments:
            self.failed = True
            return await c.close()
        if self._busy:
            raise RuntimeError("join the active group or control before issuing another operation")
        if self.failed:
            raise RuntimeError("a previous remote outcome failed; further admission is closed")
        self._busy = True
        try:
            if operation == "sample_group" and set(arguments) == {"specs"}:
                return await asyncio.to_thread(c.sample_batch, check_specs(arguments["specs"]))
            if operation == "initialize":
                if set(arguments) != {"lora_config"}:
                    raise ValueError("initialize requires the learner LoRA configuration")
                if DistributedLoRAConfig.from_dict(arguments["lora_config"]) != c.lora_config:
                    raise ValueError("learner and rollout LoRA configurations differ")
                await c.start()
                return self._status()
            if arguments:
                raise ValueError("this RPC operation accepts no JSON arguments")
            if operation == "activate" and update is not None:
                ack = await c.activate(*update)
                return {"ack": ack, "activation_receipts": copy.deepcopy(c.activation_receipts)}
            if operation in {"pause", "resume"}:
                return await getattr(c, operation)()
            raise ValueError("unknown RPC operation")
        except BaseException:
            self.failed = True
            raise
        finally:
            self._busy = False

    def server_close(self):
        super().server_close()
        if self.loop.is_running():
            self.failed = True
            try:
                asyncio.run_coroutine_threadsafe(self.controller.close(), self.loop).result(timeout=self.io_timeout)
            finally:
                self.loop.call_soon_threadsafe(self.loop.stop)
                self._thread.join(timeout=5)
                self.loop.close()


__all__ = ["RemoteLoRAClient", "RemoteLoRAServer", "check_endpoint", "check_specs", "check_token"]
