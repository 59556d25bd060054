"""JSON-RPC 2.0 handlers of barraCuda's FHE IPC methods, on this library.

barraCuda's primal server (crates/barracuda-core) exposes the FHE path as
the methods `fhe.ntt` and `fhe.pointwise_mul`
(crates/barracuda-core/src/ipc/methods/fhe.rs:11-217), over newline-
delimited JSON-RPC 2.0 on TCP or Unix sockets
(ipc/transport/connection.rs, ipc/transport/dispatch.rs, ipc/jsonrpc.rs).
This module answers the same requests with the same responses, computing
through the C ABI instead of wgpu:

  - same parameter names, checks, order of checks, error codes and message
    text (INVALID_PARAMS for missing or inconsistent parameters,
    INTERNAL_ERROR for device, setup and execution failures, with the Rust
    `Display` text of the op's error);
  - same success object {"degree", "modulus", "result", "status":
    "completed"} (keys sorted, as serde_json writes a `json!` object);
  - method names with or without the `barracuda.` prefix, unknown methods
    answered with METHOD_NOT_FOUND, notifications (no id) unanswered,
    batches as JSON arrays.

`fhe.intt` is new: the inverse transform had no IPC method.  It takes
`inv_root_of_unity` where `fhe.ntt` takes `root_of_unity` and reports
"INTT setup failed" / "INTT execution failed".
"""
from __future__ import annotations

import json
import os
import socket
import socketserver
import threading
from typing import Any, Optional

import numpy as np

from ._native import BarracudaError
from .ops import Device, FheIntt, FheNtt, FhePointwiseMul, FheTensor

PARSE_ERROR = -32700
INVALID_REQUEST = -32600
METHOD_NOT_FOUND = -32601
INVALID_PARAMS = -32602
INTERNAL_ERROR = -32603
NAMESPACE = "barracuda"
METHODS = ("fhe.ntt", "fhe.intt", "fhe.pointwise_mul")
_U32_MAX = 2**32 - 1


def _as_u64(v: Any) -> Optional[int]:
    """serde_json's Value::as_u64: a non-negative JSON integer below 2^64."""
    if isinstance(v, bool) or not isinstance(v, int):
        return None
    return v if 0 <= v < 2**64 else None


def success(id_: Any, result: Any) -> dict:
    return {"jsonrpc": "2.0", "result": result, "id": id_}


def error(id_: Any, code: int, message: str) -> dict:
    return {"jsonrpc": "2.0", "error": {"code": code, "message": message}, "id": id_}


def encode(response: Any) -> str:
    """Compact JSON, as serde_json::to_string writes it."""
    return json.dumps(response, separators=(",", ":"), ensure_ascii=False)


def normalize_method(method: str) -> str:
    """ipc/methods/mod.rs:175-180: `barracuda.fhe.ntt` is `fhe.ntt`."""
    prefix = NAMESPACE + "."
    return method[len(prefix):] if method.startswith(prefix) else method


def _upload(device: Device, poly) -> FheTensor:
    words = np.ascontiguousarray(np.asarray(poly, dtype=np.uint64)).view(np.uint32)
    return FheTensor.from_u32(words, device)


def _completed(id_, degree, modulus, tensor: FheTensor) -> dict:
    return success(id_, {"degree": degree, "modulus": modulus,
                         "result": [int(v) for v in tensor.to_u64()], "status": "completed"})


class FheIpc:
    """The FHE methods of the primal, bound to one device (None: no GPU)."""

    def __init__(self, device: Optional[Device] = None):
        self.device = device

    # ------------------------------------------------------------ methods
    def _transform(self, params: dict, id_, root_key: str, op, what: str) -> dict:
        """fhe.rs:11-106 (fhe.ntt); fhe.intt follows it with FheIntt."""
        modulus = _as_u64(params.get("modulus"))
        if modulus is None:
            return error(id_, INVALID_PARAMS, "Missing required param: modulus")
        degree = _as_u64(params.get("degree"))
        if degree is None:
            return error(id_, INVALID_PARAMS, "Missing required param: degree")
        root = _as_u64(params.get(root_key))
        if root is None:
            return error(id_, INVALID_PARAMS, f"Missing required param: {root_key}")
        coefficients = params.get("coefficients")
        if not isinstance(coefficients, list):
            return error(id_, INVALID_PARAMS, "Missing required param: coefficients")
        poly = [v for v in (_as_u64(c) for c in coefficients) if v is not None]
        if degree > _U32_MAX:
            return error(id_, INVALID_PARAMS, f"degree {degree} exceeds u32::MAX")
        if len(poly) != degree:
            return error(id_, INVALID_PARAMS, f"coefficients length {len(poly)} != degree {degree}")
        if self.device is None:
            return error(id_, INTERNAL_ERROR, "No GPU device available")
        try:
            t = _upload(self.device, poly)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Tensor creation failed: {e}")
        try:
            handle = op.new(t, degree, modulus, root)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"{what} setup failed: {e}")
        try:
            out = handle.execute()
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"{what} execution failed: {e}")
        try:
            return _completed(id_, degree, modulus, out)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Readback failed: {e}")

    def fhe_ntt(self, params: dict, id_) -> dict:
        return self._transform(params, id_, "root_of_unity", FheNtt, "NTT")

    def fhe_intt(self, params: dict, id_) -> dict:
        return self._transform(params, id_, "inv_root_of_unity", FheIntt, "INTT")

    def fhe_pointwise_mul(self, params: dict, id_) -> dict:
        """fhe.rs:108-217."""
        modulus = _as_u64(params.get("modulus"))
        if modulus is None:
            return error(id_, INVALID_PARAMS, "Missing required param: modulus")
        degree = _as_u64(params.get("degree"))
        if degree is None:
            return error(id_, INVALID_PARAMS, "Missing required param: degree")
        a_coeffs, b_coeffs = params.get("a"), params.get("b")
        if not isinstance(a_coeffs, list):
            return error(id_, INVALID_PARAMS, "Missing required param: a")
        if not isinstance(b_coeffs, list):
            return error(id_, INVALID_PARAMS, "Missing required param: b")
        a = [v for v in (_as_u64(c) for c in a_coeffs) if v is not None]
        b = [v for v in (_as_u64(c) for c in b_coeffs) if v is not None]
        if degree > _U32_MAX:
            return error(id_, INVALID_PARAMS, f"degree {degree} exceeds u32::MAX")
        if len(a) != degree or len(b) != degree:
            return error(id_, INVALID_PARAMS, f"coefficient arrays must have {degree} elements")
        if self.device is None:
            return error(id_, INTERNAL_ERROR, "No GPU device available")
        try:
            ta, tb = _upload(self.device, a), _upload(self.device, b)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Tensor creation failed: {e}")
        try:
            handle = FhePointwiseMul.new(ta, tb, degree, modulus)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Pointwise mul setup failed: {e}")
        try:
            out = handle.execute()
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Pointwise mul failed: {e}")
        try:
            return _completed(id_, degree, modulus, out)
        except BarracudaError as e:
            return error(id_, INTERNAL_ERROR, f"Readback failed: {e}")

    # ----------------------------------------------------------- dispatch
    def dispatch(self, method: str, params: Any, id_) -> dict:
        """ipc/methods/mod.rs:210-356, for the FHE methods."""
        name = normalize_method(method)
        p = params if isinstance(params, dict) else {}
        if name == "fhe.ntt":
            return self.fhe_ntt(p, id_)
        if name == "fhe.intt":
            return self.fhe_intt(p, id_)
        if name == "fhe.pointwise_mul":
            return self.fhe_pointwise_mul(p, id_)
        return error(id_, METHOD_NOT_FOUND, f"Unknown method: {method}")

    def handle_request(self, req: Any) -> Optional[dict]:
        """transport/dispatch.rs handle_request + jsonrpc.rs validate: None
        for notifications (no id, or a null id)."""
        if not isinstance(req, dict) or not isinstance(req.get("jsonrpc"), str) \
                or not isinstance(req.get("method"), str):
            return error(None, PARSE_ERROR, "Parse error")
        id_ = req.get("id")
        if req["jsonrpc"] != "2.0":
            return error(id_, INVALID_REQUEST, 'jsonrpc field must be "2.0"')
        if not req["method"]:
            return error(id_, INVALID_REQUEST, "method must not be empty")
        if id_ is None:
            return None
        return self.dispatch(req["method"], req.get("params"), id_)

    def handle_line(self, line: str) -> Optional[str]:
        """One NDJSON line in, one line out (or None): a request or a batch."""
        text = line.lstrip()
        try:
            parsed = json.loads(text)
        except ValueError:
            return encode(error(None, PARSE_ERROR, "Parse error"))
        if text.startswith("["):
            if not isinstance(parsed, list):
                return encode(error(None, PARSE_ERROR, "Parse error"))
            if not parsed:
                return encode(error(None, INVALID_REQUEST, "empty batch"))
            out = [r for r in (self.handle_request(item) for item in parsed) if r is not None]
            return encode(out) if out else None
        resp = self.handle_request(parsed)
        return encode(resp) if resp is not None else None

    # ------------------------------------------------------------- server
    def _handler(self):
        ipc = self

        class Handler(socketserver.StreamRequestHandler):
            def handle(self):
                for raw in self.rfile:
                    out = ipc.handle_line(raw.decode("utf-8", "replace"))
                    if out is not None:
                        self.wfile.write((out + "\n").encode())
                        self.wfile.flush()

        return Handler

    def serve_tcp(self, host: str = "127.0.0.1", port: int = 0) -> socketserver.ThreadingTCPServer:
        """Starts a background NDJSON server; returns it (server_address, shutdown())."""
        srv = socketserver.ThreadingTCPServer((host, port), self._handler())
        srv.daemon_threads = True
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv

    def serve_unix(self, path: str) -> socketserver.ThreadingUnixStreamServer:
        if os.path.exists(path):
            os.unlink(path)
        srv = socketserver.ThreadingUnixStreamServer(path, self._handler())
        srv.daemon_threads = True
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv


def call(address, request: Any, timeout: float = 30.0) -> Any:
    """Client helper: send one request (or batch) as an NDJSON line and read
    one response line.  `address` is (host, port) or a Unix socket path."""
    fam = socket.AF_UNIX if isinstance(address, str) else socket.AF_INET
    with socket.socket(fam, socket.SOCK_STREAM) as s:
        s.settimeout(timeout)
        s.connect(address)
        s.sendall((request if isinstance(request, str) else encode(request)).encode() + b"\n")
        buf = b""
        while not buf.endswith(b"\n"):
            chunk = s.recv(1 << 16)
            if not chunk:
                break
            buf += chunk
    return json.loads(buf) if buf.strip() else None
