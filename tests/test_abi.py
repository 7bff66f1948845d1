"""The C-ABI library loads and exports every entry point include/evelyn.h declares,
and the host-only helpers behave like the reference (no GPU needed)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import evelyn_b200 as evl
from evelyn_b200 import _native, runtime
from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "evelyn.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(evl_[a-z0-9_]+)\s*\(", text)) - {"evl_ffn_fn"})


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 40
    assert "evl_session_step" in syms and "evl_model_load" in syms


def test_library_exports_every_declared_symbol():
    lib = _native.path(runtime.LIB_NAME)
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert sorted(runtime.SIGNATURES) == declared_symbols()
    runtime.lib()  # binds every signature


def test_library_is_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", _native.path(runtime.LIB_NAME)], capture_output=True,
                         text=True).stdout
    arches = set(re.findall(r"sm_(\d+a?)", out))
    assert arches == {"100a"}, arches


def test_abi_version():
    assert runtime.lib().evl_abi_version() == 1


def test_host_argmax_log_prob_match_oracle():
    rng = np.random.default_rng(0)
    for _ in range(20):
        v = rng.standard_normal(1000).astype(np.float32)
        v[rng.integers(0, 1000)] = v.max()  # a tie
        assert evl.argmax(v) == orc.argmax(v)
        t = int(rng.integers(0, 1000))
        assert abs(evl.log_prob(v, t) - orc.log_prob(v, t)) < 1e-5
    assert evl.argmax(np.array([np.nan, 1.0], dtype=np.float32)) == 1


def test_host_argmax_edges():
    """The blocked scan keeps runtime.rs:897-905's semantics: the first maximum, NaN
    never wins, nothing above f32::MIN gives 0, ties across and inside 256-value blocks,
    ragged tails."""
    rng = np.random.default_rng(1)
    fmin = np.float32(np.finfo(np.float32).min)
    for trial in range(300):
        n = int(rng.integers(0, 1300))
        v = rng.integers(-3, 3, n).astype(np.float32)
        if trial % 5 == 0 and n:
            v[rng.integers(0, n, 3)] = np.nan
        if trial % 7 == 0:
            v[:] = -np.inf
        if trial % 11 == 0:
            v[:] = fmin
        if trial % 13 == 0 and n:
            v[rng.integers(0, n, 2)] = 7.0
        assert evl.argmax(v) == orc.argmax(v), (trial, n)
    v = np.zeros(151936, dtype=np.float32)
    v[[70000, 151935]] = 1.0
    assert evl.argmax(v) == 70000
    v[151935] = 2.0
    assert evl.argmax(v) == 151935


def test_validate_token_ids():
    evl.validate_token_ids([0, 17, 99], 100)
    with pytest.raises(evl.EvelynError) as e:
        evl.validate_token_ids([17, 100], 100)
    assert e.value.kind == "InvalidInput" and "tokenizer and GGUF match" in str(e.value)


def test_missing_model_file_is_not_found():
    with pytest.raises(evl.EvelynError) as e:
        evl.Model.load("/nonexistent/model.gguf")
    assert e.value.kind == "NotFound"


def test_model_options_defaults():
    o = runtime._Options()
    runtime.lib().evl_model_options_init(C.byref(o))
    assert o.struct_size == C.sizeof(runtime._Options) and o.device == -1 and o.tp_size == 1 and o.kv_f32 == 0
