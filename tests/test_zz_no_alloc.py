"""evl_attention_decode_noalloc: the decode attention with its split scratch in a
fixed device array. Called through the C ABI and compared with evl_attention_decode
(the allocating entry point) on the same paged KV cache, twice in a row, so a stale
error flag or stale partials left by the first call would show in the second.

The file name sorts last so the test also runs after every other GPU test."""
import numpy as np
import pytest

from evelyn_b200 import runtime

from . import gpu_util as gu

# Both entry points launch the same kernels with the same split count on the same
# inputs, so their outputs agree bit for bit.


def _case(t, hd, heads, kv_heads, seed):
    ps = 16
    rng = np.random.default_rng(seed)
    pages = (t + ps - 1) // ps
    total_pages = pages + 3
    perm = rng.permutation(total_pages)[:pages].astype(np.int32)
    kp = rng.standard_normal((total_pages, kv_heads, ps, hd)).astype(np.float16)
    vp = rng.standard_normal((total_pages, kv_heads, ps, hd)).astype(np.float16)
    q = rng.standard_normal((heads, hd)).astype(np.float32)
    return ps, gu.to_dev(q), gu.to_dev(kp), gu.to_dev(vp), gu.to_dev(perm)


def _call(fn, dq, dk, dv, dpt, t, heads, kv_heads, hd, ps):
    out = gu.empty_f32(heads * hd)
    out.fill_(float("nan"))
    runtime.check(fn(gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(dpt), t, heads, kv_heads, hd, ps, gu.ptr(out), None))
    gu.sync()
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("t,hd,heads,kv_heads", [(1, 128, 32, 8), (1000, 128, 32, 8), (3000, 64, 16, 2),
                                                 (4096, 128, 64, 8),
                                                 # the most partials any accepted shape needs: group 8
                                                 # over one kv head, one split per page up to 2 x SMs
                                                 (8192, 128, 8, 1)])
def test_noalloc_matches_allocating_entry_point(t, hd, heads, kv_heads):
    lib = runtime.lib()
    ps, dq, dk, dv, dpt = _case(t, hd, heads, kv_heads, seed=t + hd)
    want = _call(lib.evl_attention_decode, dq, dk, dv, dpt, t, heads, kv_heads, hd, ps)
    assert np.isfinite(want).all()
    for _ in range(2):
        got = _call(lib.evl_attention_decode_noalloc, dq, dk, dv, dpt, t, heads, kv_heads, hd, ps)
        assert np.array_equal(got, want)


@pytest.mark.gpu
def test_noalloc_consecutive_shapes_and_bad_input():
    lib = runtime.lib()
    # a long context, then a short one: the second must not read the first's partials
    for t, seed in ((2500, 1), (40, 2)):
        ps, dq, dk, dv, dpt = _case(t, 128, 32, 8, seed)
        want = _call(lib.evl_attention_decode, dq, dk, dv, dpt, t, 32, 8, 128, ps)
        got = _call(lib.evl_attention_decode_noalloc, dq, dk, dv, dpt, t, 32, 8, 128, ps)
        assert np.array_equal(got, want)
    # rejected before any launch: unsupported head_dim
    out = gu.empty_f32(32 * 96)
    st = lib.evl_attention_decode_noalloc(gu.ptr(dq), gu.ptr(dk), gu.ptr(dv), gu.ptr(dpt), 40, 32, 8, 96, 16,
                                          gu.ptr(out), None)
    assert st == 1 and b"head_dim" in lib.evl_last_error()
