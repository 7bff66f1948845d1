"""Kernel parity through the C ABI: exact dequantisation (bit-for-bit against the
oracle's restatement of src/gguf.rs:338-430), the repack round trip, the fused
matvec (src/runtime.rs:72-88) and paged GQA decode attention (runtime.rs:723-766)."""
import ctypes as C

import numpy as np
import pytest

from evelyn_b200 import runtime, synth
from oracle import oracle as orc
from tests import gpu_util as gu

pytestmark = pytest.mark.gpu

TYPES = [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K]
DENSE_TYPES = [synth.GGML_F32, synth.GGML_F16, synth.GGML_BF16]
BLOCK = {synth.GGML_Q8_0: 32, synth.GGML_Q4_K: 256, synth.GGML_Q5_K: 256, synth.GGML_Q6_K: 256}


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("t", TYPES)
def test_dequantize_raw_bit_exact(t):
    rng = np.random.default_rng(t)
    nblocks = 300
    raw = gu.random_blocks(t, nblocks, rng)
    n = nblocks * BLOCK[t]
    want = orc.dequantize(t, raw, n)
    d_raw = gu.to_dev(np.frombuffer(raw, dtype=np.uint8))
    d_out = gu.empty_f32(n)
    runtime.check(runtime.lib().evl_dequantize_raw(t, gu.ptr(d_raw), n, gu.ptr(d_out), None))
    gu.sync()
    got = d_out.cpu().numpy()
    assert np.array_equal(_bits(got), _bits(want))


@pytest.mark.parametrize("t", DENSE_TYPES)
def test_dequantize_raw_dense_bit_exact(t):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32)
    raw = synth.encode(t, x)
    want = orc.dequantize(t, raw, x.size)
    d_raw = gu.to_dev(np.frombuffer(raw, dtype=np.uint8))
    d_out = gu.empty_f32(x.size)
    runtime.check(runtime.lib().evl_dequantize_raw(t, gu.ptr(d_raw), x.size, gu.ptr(d_out), None))
    gu.sync()
    assert np.array_equal(_bits(d_out.cpu().numpy()), _bits(want))


def _qmatrix(t, rows, cols, raw):
    h = C.c_void_p()
    buf = np.frombuffer(raw, dtype=np.uint8)
    runtime.check(runtime.lib().evl_qmatrix_create(t, rows, cols, C.c_void_p(buf.ctypes.data), 0, C.byref(h)))
    return h


SHAPES = [(1, 256), (37, 768), (64, 4096), (33, 2304), (130, 12288 // 4)]


@pytest.mark.parametrize("t", [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K, synth.GGML_F16,
                               synth.GGML_BF16, synth.GGML_F32])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_repack_round_trip_bit_exact(t, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    if t in BLOCK:
        raw = gu.random_blocks(t, rows * cols // BLOCK[t], rng)
    else:
        raw = synth.encode(t, rng.standard_normal(rows * cols).astype(np.float32))
    want = orc.dequantize(t, raw, rows * cols)
    h = _qmatrix(t, rows, cols, raw)
    try:
        d_out = gu.empty_f32(rows * cols)
        runtime.check(runtime.lib().evl_qmatrix_dequantize(h, gu.ptr(d_out), None))
        gu.sync()
        assert np.array_equal(_bits(d_out.cpu().numpy()), _bits(want))
    finally:
        runtime.lib().evl_qmatrix_free(h)


@pytest.mark.parametrize("t", [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K, synth.GGML_F16,
                               synth.GGML_BF16, synth.GGML_F32])
@pytest.mark.parametrize("rows,cols", SHAPES + [(4096, 4096), (1000, 12288), (40, 16384)])
def test_qmatrix_matvec(t, rows, cols):
    """y = W x against the oracle's sequential f32 dot; tolerance: 5e-5 of sum|w*x| (f32 reordering).
    F16 / BF16 / F32 matrices run the warp-per-row kernel (rows of 16384 values need its
    shared-memory opt-in)."""
    rng = np.random.default_rng(rows + cols + t)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    raw = synth.encode(t, w)
    wq = orc.dequantize(t, raw, rows * cols).reshape(rows, cols).astype(np.float64)
    x = rng.standard_normal(cols).astype(np.float32)
    want = wq @ x.astype(np.float64)
    scale = np.abs(wq) @ np.abs(x.astype(np.float64))
    h = _qmatrix(t, rows, cols, raw)
    try:
        dx, dy = gu.to_dev(x), gu.empty_f32(rows)
        runtime.check(runtime.lib().evl_qmatrix_matvec(h, gu.ptr(dx), gu.ptr(dy), None))
        gu.sync()
        got = dy.cpu().numpy().astype(np.float64)
    finally:
        runtime.lib().evl_qmatrix_free(h)
    assert np.all(np.abs(got - want) <= 5e-5 * scale + 1e-7)


def _attention_ref(q, K, V, heads, kv_heads):
    hd = q.shape[-1]
    g = heads // kv_heads
    out = np.zeros((heads, hd))
    for h in range(heads):
        s = (K[:, h // g, :] @ q[h]) / np.sqrt(hd)
        w = np.exp(s - s.max())
        out[h] = (w / w.sum()) @ V[:, h // g, :]
    return out


@pytest.mark.parametrize("hd", [64, 128, 256])
@pytest.mark.parametrize("t", [1, 15, 16, 17, 100, 1000, 3000])
def test_attention_decode_paged(t, hd):
    heads, kv_heads, ps = 32, 8, 16
    rng = np.random.default_rng(t * 3 + hd)
    pages = (t + ps - 1) // ps
    total_pages = pages + 5
    perm = rng.permutation(total_pages)[:pages].astype(np.int32)  # scattered pages
    kp = rng.standard_normal((total_pages, kv_heads, ps, hd)).astype(np.float16)
    vp = rng.standard_normal((total_pages, kv_heads, ps, hd)).astype(np.float16)
    q = rng.standard_normal((heads, hd)).astype(np.float32)
    K = kp[perm].transpose(0, 2, 1, 3).reshape(pages * ps, kv_heads, hd)[:t].astype(np.float64)
    V = vp[perm].transpose(0, 2, 1, 3).reshape(pages * ps, kv_heads, hd)[:t].astype(np.float64)
    want = _attention_ref(q.astype(np.float64), K, V, heads, kv_heads)
    dq, dk, dv, dpt = gu.to_dev(q), gu.to_dev(kp), gu.to_dev(vp), gu.to_dev(perm)
    dout = gu.empty_f32(heads * hd)
    runtime.check(runtime.lib().evl_attention_decode(gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(dpt), t, heads,
                                                     kv_heads, hd, ps, gu.ptr(dout), None))
    got = dout.cpu().numpy().reshape(heads, hd)
    assert np.abs(got - want).max() < 2e-5
    # the caller-workspace variant gives the same bits
    lib = runtime.lib()
    wsb = lib.evl_attention_workspace_bytes(t + 40, heads, kv_heads, hd)
    ws = gu.torch().empty(wsb // 4 + 64, dtype=gu.torch().float32, device="cuda:0")
    wp = C.c_void_p((ws.data_ptr() + 255) // 256 * 256)
    dout2 = gu.empty_f32(heads * hd)
    runtime.check(lib.evl_attention_decode_ws(gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(dpt), t, heads, kv_heads, hd,
                                              ps, gu.ptr(dout2), wp, wsb, None))
    gu.sync()
    assert np.array_equal(dout2.cpu().numpy(), dout.cpu().numpy())
