"""Batched products on the tensor cores (evl_qmatrix_matmul, tcgen05): up to 32
vectors against one quantised matrix, checked against the float64 product of the
oracle's exact dequantisation (QMatrix::matvec, src/runtime.rs:72-88, for every
vector) and against the single-vector device matvec."""
import ctypes as C

import numpy as np
import pytest

from evelyn_b200 import runtime, synth
from oracle import oracle as orc

from . import gpu_util as gu

pytestmark = pytest.mark.gpu


def _qmatrix(t, rows, cols, raw):
    h = C.c_void_p()
    buf = np.frombuffer(raw, dtype=np.uint8)
    runtime.check(runtime.lib().evl_qmatrix_create(t, rows, cols, C.c_void_p(buf.ctypes.data), 0, C.byref(h)))
    return h


@pytest.mark.parametrize("t", [synth.GGML_Q4_K, synth.GGML_Q6_K, synth.GGML_Q8_0])
@pytest.mark.parametrize("rows,cols,nvec", [(128, 256, 1), (300, 512, 5), (1000, 1024, 32), (4096, 4096, 8),
                                            (200, 3072, 17)])
def test_matmul_matches_float64(t, rows, cols, nvec):
    rng = np.random.default_rng(rows * 3 + cols + nvec + t)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    raw = synth.encode(t, w)
    wq = orc.dequantize(t, raw, rows * cols).reshape(rows, cols).astype(np.float64)
    x = rng.standard_normal((nvec, cols)).astype(np.float32)
    x[0, :17] *= 30.0  # one outlier-heavy vector
    want = x.astype(np.float64) @ wq.T
    scale = np.abs(x.astype(np.float64)) @ np.abs(wq.T)
    h = _qmatrix(t, rows, cols, raw)
    try:
        dx, dy = gu.to_dev(x), gu.empty_f32(nvec * rows)
        runtime.check(runtime.lib().evl_qmatrix_matmul(h, gu.ptr(dx), nvec, gu.ptr(dy), None))
        got = dy.cpu().numpy().reshape(nvec, rows).astype(np.float64)
        # the single-vector path on the same data
        dv = gu.empty_f32(rows)
        runtime.check(runtime.lib().evl_qmatrix_matvec(h, gu.ptr(dx[nvec - 1]), gu.ptr(dv), None))
        gu.sync()
        one = dv.cpu().numpy().astype(np.float64)
    finally:
        runtime.lib().evl_qmatrix_free(h)
    err = np.abs(got - want)
    assert np.all(err <= 5e-5 * scale + 1e-7), float((err / (scale + 1e-12)).max())
    assert np.all(np.abs(got[nvec - 1] - one) <= 1e-4 * scale[nvec - 1] + 1e-7)


def test_matmul_repeat_and_errors():
    t, rows, cols = synth.GGML_Q4_K, 256, 512
    rng = np.random.default_rng(5)
    raw = synth.encode(t, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    h = _qmatrix(t, rows, cols, raw)
    try:
        x = rng.standard_normal((4, cols)).astype(np.float32)
        dx = gu.to_dev(x)
        outs = []
        for _ in range(2):
            dy = gu.empty_f32(4 * rows)
            runtime.check(runtime.lib().evl_qmatrix_matmul(h, gu.ptr(dx), 4, gu.ptr(dy), None))
            outs.append(dy.cpu().numpy())
        assert np.array_equal(outs[0], outs[1])  # deterministic (fixed-order split reduction)
        assert runtime.lib().evl_qmatrix_matmul(h, gu.ptr(dx), 33, gu.ptr(dy), None) == 1
    finally:
        runtime.lib().evl_qmatrix_free(h)
