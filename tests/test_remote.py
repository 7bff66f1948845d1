"""The AARNN routing bridge (src/remote.rs) against fake knowledge regions on loopback:
the wire format (:69-111), one reconnect (:114-143), non-finite / width / status
errors turning into a dense fallback with a counter (:247-271), and the endpoint
stats (:13-24, :145-154). Failures are made on the host (a server that drops,
answers wrongly or goes away); no GPU is involved."""
import ctypes as C
import socket
import struct
import threading

import numpy as np
import pytest

from evelyn_b200 import runtime

EVL_FFN_DENSE = 1


class FakeRegion:
    """A TCP server speaking the region protocol; `mode` picks its behaviour per request."""

    def __init__(self, modes):
        self.modes = list(modes)
        self.sock = socket.socket()
        self.sock.bind(("127.0.0.1", 0))
        self.sock.listen(8)
        self.port = self.sock.getsockname()[1]
        self.requests = 0
        self.connections = 0
        self.thread = threading.Thread(target=self.serve, daemon=True)
        self.thread.start()

    def serve(self):
        while True:
            try:
                conn, _ = self.sock.accept()
            except OSError:
                return
            self.connections += 1
            try:
                self._session(conn)
            except OSError:
                pass

    def _session(self, conn):
        with conn:
            if True:
                while True:
                    hdr = self._read(conn, 4)
                    if hdr is None:
                        break
                    (w,) = struct.unpack("<I", hdr)
                    x = np.frombuffer(self._read(conn, 4 * w), dtype="<f4")
                    mode = self.modes.pop(0) if self.modes else "ok"
                    self.requests += 1
                    if mode == "drop":
                        break
                    if mode == "status":
                        conn.sendall(struct.pack("<II", 7, w))
                        continue
                    if mode == "width":
                        conn.sendall(struct.pack("<II", 0, w - 1) + (2 * x[:-1]).astype("<f4").tobytes())
                        continue
                    y = 2 * x
                    if mode == "nan":
                        y = y.copy()
                        y[0] = np.nan
                    conn.sendall(struct.pack("<II", 0, w) + y.astype("<f4").tobytes())

    @staticmethod
    def _read(conn, n):
        buf = b""
        while len(buf) < n:
            chunk = conn.recv(n - len(buf))
            if not chunk:
                return None
            buf += chunk
        return buf

    def close(self):
        self.sock.close()


def make_remote(layers_addrs, timeout_ms=2000):
    lib = runtime.lib()
    items = sorted(layers_addrs.items())
    ids = (C.c_size_t * len(items))(*[k for k, _ in items])
    keep = [a.encode() for _, a in items]
    addrs = (C.c_char_p * len(items))(*keep)
    h = C.c_void_p()
    runtime.check(lib.evl_remote_ffn_new(None, len(items), ids, addrs, timeout_ms, C.byref(h)))
    b = runtime._Backend()
    runtime.check(lib.evl_remote_ffn_backend(h, C.byref(b)))
    return h, b


def call(b, layer, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros_like(x)
    rc = b.ffn(b.ctx, layer, x.ctypes.data_as(C.POINTER(C.c_float)), x.size, y.ctypes.data_as(C.POINTER(C.c_float)))
    return rc, y


def stats(h, layer):
    st = runtime._EndpointStats()
    runtime.check(runtime.lib().evl_remote_ffn_stats(h, layer, C.byref(st)))
    return st


def test_round_trip_and_persistent_connection():
    srv = FakeRegion(["ok"] * 3)
    h, b = make_remote({2: f"127.0.0.1:{srv.port}"})
    try:
        x = np.arange(16, dtype=np.float32)
        for _ in range(3):
            rc, y = call(b, 2, x)
            assert rc == 0 and np.array_equal(y, 2 * x)
        assert srv.connections == 1  # one persistent stream
        st = stats(h, 2)
        assert st.calls == 3 and st.failures == 0 and st.retries == 0 and st.max_ns > 0
        assert runtime.lib().evl_remote_ffn_fallbacks(h) == 0
        assert list(b.routed[:3]) == [0, 0, 1]
        # a layer with no region is dense
        rc, _ = call(b, 0, x)
        assert rc == EVL_FFN_DENSE
    finally:
        runtime.lib().evl_remote_ffn_free(h)
        srv.close()


def test_dropped_connection_reconnects_once():
    srv = FakeRegion(["drop", "ok"])
    h, b = make_remote({0: f"127.0.0.1:{srv.port}"})
    try:
        x = np.ones(8, dtype=np.float32)
        rc, y = call(b, 0, x)
        assert rc == 0 and np.array_equal(y, 2 * x)
        st = stats(h, 0)
        assert st.retries == 1 and st.failures == 0 and srv.connections == 2
    finally:
        runtime.lib().evl_remote_ffn_free(h)
        srv.close()


@pytest.mark.parametrize("mode", ["status", "width", "nan"])
def test_bad_answers_fall_back_to_dense(mode):
    srv = FakeRegion([mode, mode])  # both attempts fail
    h, b = make_remote({1: f"127.0.0.1:{srv.port}"})
    try:
        rc, _ = call(b, 1, np.ones(8, dtype=np.float32))
        assert rc == EVL_FFN_DENSE
        assert runtime.lib().evl_remote_ffn_fallbacks(h) == 1
        st = stats(h, 1)
        assert st.calls == 1 and st.failures == 1 and st.retries == 1
    finally:
        runtime.lib().evl_remote_ffn_free(h)
        srv.close()


def test_unreachable_region_falls_back():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()  # nothing listens here
    h, b = make_remote({0: f"127.0.0.1:{port}"})
    try:
        rc, _ = call(b, 0, np.ones(4, dtype=np.float32))
        assert rc == EVL_FFN_DENSE
        assert runtime.lib().evl_remote_ffn_fallbacks(h) == 1
        assert stats(h, 0).failures == 1
    finally:
        runtime.lib().evl_remote_ffn_free(h)


def test_stats_for_unrouted_layer_is_not_found():
    h, b = make_remote({3: "127.0.0.1:1"})
    try:
        st = runtime._EndpointStats()
        rc = runtime.lib().evl_remote_ffn_stats(h, 1, C.byref(st))
        assert rc == 3  # NotFound
    finally:
        runtime.lib().evl_remote_ffn_free(h)


def test_zero_read_timeout_falls_back():
    """set_read_timeout(Some(Duration::ZERO)) fails in the reference's connect
    (remote.rs:62-64), so the layer falls back to the dense FFN instead of blocking."""
    srv = FakeRegion(["ok"] * 4)
    h, b = make_remote({0: f"127.0.0.1:{srv.port}"}, timeout_ms=0)
    try:
        rc, _ = call(b, 0, np.ones(4, dtype=np.float32))
        assert rc == EVL_FFN_DENSE
        assert runtime.lib().evl_remote_ffn_fallbacks(h) == 1
        st = stats(h, 0)
        assert st.failures == 1 and st.retries == 1 and srv.requests == 0
    finally:
        runtime.lib().evl_remote_ffn_free(h)
        srv.close()
