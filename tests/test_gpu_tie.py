"""Exact argmax ties on the GPU: among equal maximal logits the engine picks
the last index, as the reference's Iterator::max_by(f32::total_cmp) does
(crates/needle-infer/src/engine.rs:299-304).  Two embedding rows are made
identical, so the tied head gives both tokens bit-identical logits, and the
step mask allows only those two: every step must emit the higher index.
Covered on the CUDA-core head (one request) and on the tensor-core head's
mask + argmax epilogue (a 160-request batch)."""
import json
import struct

import numpy as np
import pytest

import oracle as orc
from conftest import load_pkg

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")
LO, HI = 100, 2000  # the tied pair; HI is the last maximal index


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def tied_model():
    blob = bytearray(wl.random_model(seed=23, num_encoder_layers=2, num_decoder_layers=2))
    hl = struct.unpack("<Q", bytes(blob[:8]))[0]
    hdr = json.loads(bytes(blob[8:8 + hl]))
    e = hdr["embedding"]
    assert e["dtype"] == "BF16"
    d = e["shape"][1]
    base = 8 + hl + e["data_offsets"][0]
    row = lambda r: slice(base + 2 * d * r, base + 2 * d * (r + 1))  # noqa: E731
    blob[row(HI)] = blob[row(LO)]
    return bytes(blob)


def pair_masks(n_req, steps):
    m = np.zeros((n_req, steps, 128), np.uint64)
    m[:, :, LO // 64] |= np.uint64(1 << (LO % 64))
    m[:, :, HI // 64] |= np.uint64(1 << (HI % 64))
    return m


@pytest.fixture(scope="module")
def tied():
    blob = tied_model()
    return nb.NeedleEngine.from_bytes(blob, "a\nb\n"), orc.Model(data=blob)


def test_tie_picks_last_index_single_request(tied):
    eng, ref = tied
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, 8192, 37)
    masks = pair_masks(1, 4)
    ids, lens, lg = eng.run_batch_ids([prompt], 4, mask_bits=masks, want_logits=True)
    assert np.all(lg[0, :, LO] == lg[0, :, HI])  # bit-identical tied logits
    assert ids[0].tolist() == [HI] * 4
    rid, _ = ref.generate(prompt, 4, mask_bits=masks[0])
    assert rid.tolist() == [HI] * 4


def test_tie_picks_last_index_tensor_core_head(tied):
    eng, ref = tied
    ids_in, off = wl.random_prompts(160, 8, 64, 8192, seed=2)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(160)]
    masks = pair_masks(160, 3)
    ids, lens, lg = eng.run_batch_ids(prompts, 3, mask_bits=masks, want_logits=True)
    assert np.all(lg[:, :, LO] == lg[:, :, HI])
    assert np.all(ids == HI)
    rid, _ = ref.generate(prompts[7], 3, mask_bits=masks[7])
    assert rid.tolist() == [HI] * 3
