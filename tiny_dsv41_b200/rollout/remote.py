"""Private-network LoRA rollout RPC: authenticated JSON frames plus raw tensor packets, never pickle.

The wire protocol is the one the rollout service speaks (``rollout_manager/backends/
vllm_lora_remote.py:96-346``), so a learner here drives that vLLM service and this library's
native service (``rollout.native_service``) alike:

* one TCP connection per call; each JSON message is a 4-byte big-endian length and at most
  32 MiB of compact JSON with finite numbers only;
* authentication first: the client sends ``{"token": ...}`` (32..256 characters of
  [A-Za-z0-9_-]), the server answers ``{"authenticated": true | false}`` after a constant-time
  comparison;
* then ``{"operation": ..., "arguments": {...}}`` (initialize, status, activate, sample_group,
  pause, resume, close); ``activate`` is followed by one LoRA update frame of
  ``rollout.lora_transport``, read only after authentication;
* the answer is ``{"ok": true, "result": ...}`` or ``{"ok": false, "error": ..., ...}``.

Endpoints must be private or loopback IPv4 addresses. Both ends latch failure: after any error a
client allows only status and close (an unknown outcome is never retried) and a server admits
nothing but status and close. ``sample_group`` takes 1..32 specs ``{prompt_ids, max_tokens,
temperature, request_id (32 hex), sampling_seed}``.
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
from contextlib import contextmanager

from ..rl.lora_config import DistributedLoRAConfig
from .lora_transport import _read_exact, receive_update, send_update

MAX_JSON_BYTES = 32 << 20
AUTH_BYTES = 4096
MAX_TIMEOUT = 7200
OPERATIONS = {"initialize", "status", "activate", "sample_group", "pause", "resume", "close"}
ALWAYS_ALLOWED = {"status", "close"}
_PRIVATE_NETWORKS = tuple(ipaddress.ip_network(n) for n in ("10.0.0.0/8", "172.16.0.0/12", "192.168.0.0/16",
                                                            "127.0.0.0/8"))
_TOKEN = re.compile(r"[A-Za-z0-9_-]{32,256}")
_REQUEST_ID = re.compile(r"[0-9a-f]{32}")
_LENGTH = struct.Struct("!I")


def check_endpoint(address) -> tuple[str, int]:
    host, port = address
    ip = ipaddress.IPv4Address(host)
    private = any(ip in network for network in _PRIVATE_NETWORKS)
    if not (private and type(port) is int and 0 <= port <= 65535):
        raise ValueError("RPC requires an explicit private or loopback IPv4 address and valid port")
    return str(ip), port


def check_token(value) -> str:
    if isinstance(value, str) and _TOKEN.fullmatch(value):
        return value
    raise ValueError("RPC token requires 32..256 ASCII letters, digits, underscores or hyphens")


def _check_timeout(value, what: str) -> float:
    if type(value) in (int, float) and math.isfinite(value) and 0 < value <= MAX_TIMEOUT:
        return value
    raise ValueError(f"{what} must be finite and at most 7200 seconds")


# -- framing ----------------------------------------------------------------------------------------
def send_json(stream, value) -> None:
    body = json.dumps(value, separators=(",", ":"), allow_nan=False).encode()
    if not 0 < len(body) <= MAX_JSON_BYTES:
        raise ValueError("RPC JSON exceeds byte budget")
    stream.sendall(_LENGTH.pack(len(body)) + body)


def _no_constants(_name):
    raise ValueError("RPC JSON requires finite values")


def receive_json(stream, limit: int = MAX_JSON_BYTES):
    (size,) = _LENGTH.unpack(_read_exact(stream, _LENGTH.size))
    if not 0 < size <= limit:
        raise ValueError("RPC JSON exceeds byte budget")
    return json.loads(_read_exact(stream, size), parse_constant=_no_constants)


# -- sample request validation ----------------------------------------------------------------------
_SPEC_RULES = {
    "prompt_ids": lambda v: (isinstance(v, list) and 1 <= len(v) <= 4096
                             and all(type(t) is int and 0 <= t < 2 ** 31 for t in v)),
    "max_tokens": lambda v: type(v) is int and 1 <= v <= 4096,
    "temperature": lambda v: type(v) in (int, float) and math.isfinite(v) and 0 < v <= 10,
    "request_id": lambda v: isinstance(v, str) and _REQUEST_ID.fullmatch(v) is not None,
    "sampling_seed": lambda v: type(v) is int and 0 <= v < 2 ** 63 - 1,
}


def check_specs(values):
    if not (isinstance(values, list) and 1 <= len(values) <= 32):
        raise ValueError("sample_group requires 1..32 request specifications")
    request_ids = set()
    for spec in values:
        if not isinstance(spec, dict) or spec.keys() != _SPEC_RULES.keys():
            raise ValueError("invalid sample request fields")
        if not all(rule(spec[name]) for name, rule in _SPEC_RULES.items()) or spec["request_id"] in request_ids:
            raise ValueError("invalid bounded sample request or duplicate request ID")
        request_ids.add(spec["request_id"])
    return values


# -- client -----------------------------------------------------------------------------------------
def _failure_detail(response) -> str:
    if not isinstance(response, dict):
        return "invalid response; outcome unknown"
    return f"{response.get('error_type', 'UnknownError')}: {response.get('reason', 'outcome unknown')}"


class RemoteLoRAClient:
    """Synchronous client; the first error latches failure (only status and close stay allowed)."""

    def __init__(self, host, port, token, *, timeout: float = 7200) -> None:
        self.address = check_endpoint((host, port))
        self._token = check_token(token)
        self.timeout = _check_timeout(timeout, "RPC timeout")
        self.failed = self.closed = False
        self._lock = threading.Lock()
        self.ack = self.activation_receipts = self.base_identity = None

    @contextmanager
    def _authenticated(self):
        with socket.create_connection(self.address, timeout=self.timeout) as stream:
            send_json(stream, {"token": self._token})
            if receive_json(stream, AUTH_BYTES) != {"authenticated": True}:
                raise PermissionError("remote authentication rejected")
            yield stream

    def _call(self, operation, arguments=None, update=None):
        if operation not in OPERATIONS:
            raise ValueError("unknown RPC operation")
        with self._lock:
            if self.closed or (self.failed and operation not in ALWAYS_ALLOWED):
                raise RuntimeError("remote client has a closed or unknown prior outcome; no retry is allowed")
            try:
                with self._authenticated() as stream:
                    send_json(stream, {"operation": operation, "arguments": arguments or {}})
                    if update is not None:
                        send_update(stream, *update)
                    response = receive_json(stream)
                if isinstance(response, dict) and response.get("ok") is True and "result" in response:
                    return response["result"]
                raise RuntimeError(f"remote {operation} failed: {_failure_detail(response)}")
            except BaseException:
                self.failed = True
                raise

    def initialize(self, *, lora_config=None):
        profile = DistributedLoRAConfig() if lora_config is None else DistributedLoRAConfig.from_dict(lora_config)
        result = self._call("initialize", {"lora_config": profile.to_dict()})
        try:
            served = DistributedLoRAConfig.from_dict(result["lora_config"])
            identity = result["base_identity"]
        except (KeyError, TypeError, ValueError) as error:
            self.failed = True
            raise RuntimeError("remote initialize returned an invalid LoRA configuration") from error
        if served != profile:
            self.failed = True
            raise RuntimeError("remote initialize returned an invalid LoRA configuration") from ValueError(
                "rollout LoRA configuration differs from the learner profile")
        self.base_identity = identity
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


# -- server -----------------------------------------------------------------------------------------
def _valid_auth(message, token: str) -> bool:
    return (isinstance(message, dict) and set(message) == {"token"} and isinstance(message["token"], str)
            and hmac.compare_digest(message["token"].encode(), token.encode()))


def _valid_envelope(message) -> bool:
    return (isinstance(message, dict) and set(message) == {"operation", "arguments"}
            and message["operation"] in OPERATIONS and isinstance(message["arguments"], dict))


class _Handler(socketserver.BaseRequestHandler):
    def handle(self):
        server, stream = self.server, self.request
        authenticated, operation = False, "authentication"
        try:
            stream.settimeout(5)
            if not _valid_auth(receive_json(stream, AUTH_BYTES), server.token):
                send_json(stream, {"authenticated": False})
                return
            send_json(stream, {"authenticated": True})
            authenticated = True
            stream.settimeout(server.io_timeout)
            request = receive_json(stream)
            if not _valid_envelope(request):
                raise ValueError("invalid RPC request envelope")
            operation = request["operation"]
            update = receive_update(stream) if operation == "activate" else None
            work = asyncio.run_coroutine_threadsafe(server.dispatch(operation, request["arguments"], update),
                                                    server.loop)
            send_json(stream, {"ok": True, "result": work.result(timeout=server.io_timeout)})
        except Exception as error:
            self._reject(error, authenticated, operation)

    def _reject(self, error, authenticated: bool, operation: str) -> None:
        server = self.server
        response = {"ok": False, "error": "remote operation rejected or outcome unknown"}
        if authenticated:  # details only for an authenticated peer, never the token itself
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

    The controller provides coroutines ``start()``, ``activate(manifest, payload) -> ack``,
    ``pause()``, ``resume()``, ``close()``, a blocking ``sample_batch(specs) -> results``, and the
    attributes ``state``, ``ack``, ``base_identity``, ``lora_config``, ``activation_receipts``.
    At most 8 connections are served at a time and one operation other than status / close."""

    daemon_threads = True
    request_queue_size = 8

    def __init__(self, address, token, controller, *, io_timeout: float = 7200) -> None:
        address = check_endpoint(address)
        self.token = check_token(token)
        self.io_timeout = _check_timeout(io_timeout, "server RPC timeout")
        self.controller = controller
        self.failed = False
        self._connections = threading.BoundedSemaphore(8)
        self._busy = False
        super().__init__(address, _Handler)
        self.loop = asyncio.new_event_loop()
        self._thread = threading.Thread(target=self.loop.run_forever, daemon=True)
        self._thread.start()

    def process_request(self, request, client_address):
        if not self._connections.acquire(blocking=False):
            self.shutdown_request(request)  # over the connection limit: drop
            return
        try:
            super().process_request(request, client_address)
        except BaseException:
            self._connections.release()
            raise

    def process_request_thread(self, request, client_address):
        try:
            super().process_request_thread(request, client_address)
        finally:
            self._connections.release()

    def _status(self) -> dict:
        c = self.controller
        return {"state": c.state, "failed": self.failed or c.state == "failed", "policy_ack": copy.deepcopy(c.ack),
                "base_identity": copy.deepcopy(c.base_identity), "lora_config": c.lora_config.to_dict(),
                "activation_receipts": copy.deepcopy(c.activation_receipts)}

    async def _initialize(self, arguments):
        if set(arguments) != {"lora_config"}:
            raise ValueError("initialize requires the learner LoRA configuration")
        if DistributedLoRAConfig.from_dict(arguments["lora_config"]) != self.controller.lora_config:
            raise ValueError("learner and rollout LoRA configurations differ")
        await self.controller.start()
        return self._status()

    async def _admitted(self, operation, arguments, update):
        c = self.controller
        if operation == "sample_group" and set(arguments) == {"specs"}:
            return await asyncio.to_thread(c.sample_batch, check_specs(arguments["specs"]))
        if operation == "initialize":
            return await self._initialize(arguments)
        if arguments:
            raise ValueError("this RPC operation accepts no JSON arguments")
        if operation == "activate" and update is not None:
            ack = await c.activate(*update)
            return {"ack": ack, "activation_receipts": copy.deepcopy(c.activation_receipts)}
        if operation in ("pause", "resume"):
            return await getattr(c, operation)()
        raise ValueError("unknown RPC operation")

    async def dispatch(self, operation, arguments, update):
        if operation == "status" and not arguments:
            return self._status()
        if operation == "close" and not arguments:
            self.failed = True
            return await self.controller.close()
        if self._busy:
            raise RuntimeError("join the active group or control before issuing another operation")
        if self.failed:
            raise RuntimeError("a previous remote outcome failed; further admission is closed")
        self._busy = True
        try:
            return await self._admitted(operation, arguments, update)
        except BaseException:
            self.failed = True
            raise
        finally:
            self._busy = False

    def server_close(self):
        super().server_close()
        if not self.loop.is_running():
            return
        self.failed = True
        try:
            asyncio.run_coroutine_threadsafe(self.controller.close(), self.loop).result(timeout=self.io_timeout)
        finally:
            self.loop.call_soon_threadsafe(self.loop.stop)
            self._thread.join(timeout=5)
            self.loop.close()


__all__ = ["RemoteLoRAClient", "RemoteLoRAServer", "check_endpoint", "check_specs", "check_token"]
