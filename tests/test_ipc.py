"""CPU tests of the JSON-RPC FHE methods (barracuda_b200.ipc) without a
device: parameter checks, error codes and text, method names, notifications,
batches and the NDJSON transport, as crates/barracuda-core's handler tests
(ipc/methods_tests/tensor_fhe_tests.rs, comprehensive_tests.rs) expect."""
import json

import pytest

from barracuda_b200 import ipc

NTT = {"modulus": 17, "degree": 4, "root_of_unity": 4, "coefficients": [1, 2, 3, 4]}
PMUL = {"modulus": 17, "degree": 4, "a": [1, 2, 3, 4], "b": [5, 6, 7, 8]}


def _err(resp):
    return resp["error"]["code"], resp["error"]["message"]


@pytest.mark.parametrize("drop,msg", [("modulus", "Missing required param: modulus"),
                                      ("degree", "Missing required param: degree"),
                                      ("root_of_unity", "Missing required param: root_of_unity"),
                                      ("coefficients", "Missing required param: coefficients")])
def test_ntt_missing_params(drop, msg):
    p = {k: v for k, v in NTT.items() if k != drop}
    assert _err(ipc.FheIpc().dispatch("fhe.ntt", p, 170)) == (ipc.INVALID_PARAMS, msg)


def test_ntt_checks_and_no_device():
    h = ipc.FheIpc()
    assert _err(h.dispatch("fhe.ntt", {}, 18)) == (ipc.INVALID_PARAMS, "Missing required param: modulus")
    p = dict(NTT, coefficients=[1, 2, 3])
    assert _err(h.dispatch("fhe.ntt", p, 1)) == (ipc.INVALID_PARAMS, "coefficients length 3 != degree 4")
    # non-integer entries are dropped before the length check (filter_map(as_u64))
    p = dict(NTT, coefficients=[1, 2, "x", 3.0, 4, True, -1])
    assert _err(h.dispatch("fhe.ntt", p, 1)) == (ipc.INVALID_PARAMS, "coefficients length 3 != degree 4")
    p = dict(NTT, degree=2**32, coefficients=[])
    assert _err(h.dispatch("fhe.ntt", p, 1)) == (ipc.INVALID_PARAMS, "degree 4294967296 exceeds u32::MAX")
    assert _err(h.dispatch("fhe.ntt", NTT, 17)) == (ipc.INTERNAL_ERROR, "No GPU device available")
    # float and negative numbers are not u64
    assert _err(h.dispatch("fhe.ntt", dict(NTT, modulus=17.0), 1))[1] == "Missing required param: modulus"
    assert _err(h.dispatch("fhe.ntt", dict(NTT, degree=-4), 1))[1] == "Missing required param: degree"


def test_intt_and_pointwise_checks():
    h = ipc.FheIpc()
    p = {"modulus": 17, "degree": 4, "inv_root_of_unity": 13, "coefficients": [1, 2, 3, 4]}
    assert _err(h.dispatch("fhe.intt", dict(p, inv_root_of_unity=None), 1)) == (
        ipc.INVALID_PARAMS, "Missing required param: inv_root_of_unity")
    assert _err(h.dispatch("fhe.intt", p, 1)) == (ipc.INTERNAL_ERROR, "No GPU device available")
    assert _err(h.dispatch("fhe.pointwise_mul", {k: v for k, v in PMUL.items() if k != "a"}, 180)) == (
        ipc.INVALID_PARAMS, "Missing required param: a")
    assert _err(h.dispatch("fhe.pointwise_mul", {k: v for k, v in PMUL.items() if k != "b"}, 181)) == (
        ipc.INVALID_PARAMS, "Missing required param: b")
    assert _err(h.dispatch("fhe.pointwise_mul", dict(PMUL, b=[1]), 1)) == (
        ipc.INVALID_PARAMS, "coefficient arrays must have 4 elements")
    assert _err(h.dispatch("fhe.pointwise_mul", PMUL, 19)) == (ipc.INTERNAL_ERROR, "No GPU device available")


def test_method_names_and_envelope():
    h = ipc.FheIpc()
    r = h.dispatch("barracuda.fhe.ntt", NTT, 207)
    assert r["id"] == 207 and r["jsonrpc"] == "2.0" and "result" not in r
    assert _err(h.dispatch("fhe.nope", {}, 3)) == (ipc.METHOD_NOT_FOUND, "Unknown method: fhe.nope")
    # notification: no response
    assert h.handle_line(json.dumps({"jsonrpc": "2.0", "method": "fhe.ntt", "params": NTT})) is None
    assert json.loads(h.handle_line("{not json")) == ipc.error(None, ipc.PARSE_ERROR, "Parse error")
    r = json.loads(h.handle_line(json.dumps({"jsonrpc": "1.0", "method": "fhe.ntt", "id": 5})))
    assert _err(r) == (ipc.INVALID_REQUEST, 'jsonrpc field must be "2.0"') and r["id"] == 5
    assert json.loads(h.handle_line("[]")) == ipc.error(None, ipc.INVALID_REQUEST, "empty batch")
    batch = [{"jsonrpc": "2.0", "method": "fhe.ntt", "params": {}, "id": 1},
             {"jsonrpc": "2.0", "method": "fhe.ntt", "params": NTT},  # notification
             {"jsonrpc": "2.0", "method": "fhe.pointwise_mul", "params": PMUL, "id": 2}]
    out = json.loads(h.handle_line(json.dumps(batch)))
    assert [o["id"] for o in out] == [1, 2]
    # compact serialization, fields in the Rust struct order
    assert h.handle_line('{"jsonrpc":"2.0","method":"x","id":9}') == \
        '{"jsonrpc":"2.0","error":{"code":-32601,"message":"Unknown method: x"},"id":9}'


def test_tcp_transport_roundtrip():
    srv = ipc.FheIpc().serve_tcp("127.0.0.1", 0)
    try:
        r = ipc.call(srv.server_address, {"jsonrpc": "2.0", "method": "fhe.ntt", "params": NTT, "id": 1})
        assert _err(r) == (ipc.INTERNAL_ERROR, "No GPU device available")
    finally:
        srv.shutdown()
        srv.server_close()
