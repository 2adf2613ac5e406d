"""Host-side checks that need no GPU: the C-ABI library loads and exports
every symbol of include/*.h, NULL / error conventions of
crates/needle-c/src/lib.rs, request sharding, and the synthetic workload."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import oracle as orc
from conftest import ROOT, load_pkg

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")


def declared_functions():
    names = set()
    for h in ("needle.h", "needle_b200.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(needle_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 10 + 20
    L = nb.lib()
    missing = [n for n in sorted(names) if not hasattr(L, n)]
    assert not missing, missing
    for n in ("needle_load", "needle_load_bytes", "needle_run", "needle_run_stream", "needle_contrastive_dim",
              "needle_encode_contrastive", "needle_retrieve_tools", "needle_free_str", "needle_free",
              "needle_last_error"):
        assert n in names


def test_null_handle_conventions():
    L = nb.lib()
    # lib.rs:81-83: a NULL handle yields NULL and no error.
    assert L.needle_run(None, b"q", b"[]") is None
    assert L.needle_contrastive_dim(None) == 0
    assert not L.needle_encode_contrastive(None, b"x", None, 0)
    L.needle_free(None)
    L.needle_free_str(None)
    assert L.needle_load_bytes(None, 0, None, 0) is None
    assert nb.last_error() == "null pointer passed to needle_load_bytes"


def test_load_error_sets_message():
    L = nb.lib()
    assert L.needle_load(b"/nonexistent/w.safetensors", b"/nonexistent/v.txt") is None
    assert nb.last_error().startswith("load error:")


def test_shard_requests_balances():
    ids, off = wl.random_prompts(1000, 64, 512, 8192, seed=3)
    a = nb.shard_requests(off, 8)
    assert a.min() == 0 and a.max() == 7
    T = np.diff(off).astype(np.float64)
    cost = T * T + 2048 * T
    loads = np.array([cost[a == s].sum() for s in range(8)])
    assert loads.max() / loads.min() < 1.01


def test_pack_codes_matches_oracle_unpacking():
    rng = np.random.default_rng(0)
    codes = rng.integers(-8, 8, size=(64, 24))
    scales = rng.uniform(0.005, 0.02, size=(2, 24)).astype(np.float32)
    deq = orc.dequantize(wl.pack_codes(codes), scales, 64, 24)
    want = codes.astype(np.float32) * np.repeat(scales, 32, axis=0)
    assert np.array_equal(deq, want)


def test_random_model_loads_in_oracle():
    blob = wl.random_model(seed=1, num_encoder_layers=1, num_decoder_layers=1, vocab_size=256)
    m = orc.Model(data=blob)
    assert m.cfg["d_model"] == 512 and m.cfg["vocab_size"] == 256 and m.cfg["num_layers"] == 1


def test_random_masks_density_and_forced():
    mb = wl.random_masks(8, 4, 8192, frac=0.05, seed=2)
    bits = np.unpackbits(mb.view(np.uint8), axis=-1, bitorder="little")[..., :8192]
    assert bits.sum(axis=-1).min() >= 1
    assert abs(bits.mean() - 0.05) < 0.005
