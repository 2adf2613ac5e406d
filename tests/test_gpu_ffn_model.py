"""Checkpoints with feed-forward blocks (no_feedforward = false,
crates/needle-infer/src/engine.rs:679-707; layers.rs:46-149 with ffn.rs:19-56
in every encoder and decoder layer) against the oracle, for each activation
(drelu, swiglu, geglu).  The batched case (192 requests) runs the gate/up
projection as a tensor-core GEMM whose epilogue applies the activation; the
single request runs the CUDA-core matvec path.

Logits and token ids are held to the parity bar (1e-4 + 1e-3 |ref|).  The
encoder output of swiglu / geglu models is badly conditioned: relative noise
of 4e-6 on the oracle's own F32 weights (about the per-product precision of
the tensor cores' three-term bf16 split) moves the oracle's encoder output by
up to ~1e-3 while its logits move by ~1e-5.  The encoder output is therefore
checked against that measured sensitivity: within 3x the oracle's own
deviation under such noise."""
import json
import struct

import numpy as np
import pytest

import oracle as orc
from conftest import ATOL, RTOL, load_pkg

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")


def perturbed(blob, rel, seed):
    """The SafeTensors bytes with every F32 tensor scaled by (1 + rel * N(0,1))."""
    n = struct.unpack("<Q", blob[:8])[0]
    hdr = json.loads(blob[8:8 + n])
    base, b, rng = 8 + n, bytearray(blob), np.random.default_rng(seed)
    for name, t in hdr.items():
        if name == "__metadata__" or t["dtype"] != "F32":
            continue
        s, e = t["data_offsets"]
        a = np.frombuffer(bytes(b[base + s:base + e]), np.float32).copy()
        a *= (1 + rel * rng.standard_normal(a.shape)).astype(np.float32)
        b[base + s:base + e] = a.tobytes()
    return bytes(b)


def close(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.all(np.abs(got - ref) <= ATOL + RTOL * np.abs(ref))


@pytest.fixture(scope="module", params=["drelu", "swiglu", "geglu"])
def ffn_model(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    blob = wl.random_model(seed=40, no_feedforward=False, activation=request.param, num_encoder_layers=3,
                           num_decoder_layers=2, max_dec_len=16)
    eng = nb.NeedleEngine.from_bytes(blob, "a\nb\n")
    yield eng, orc.Model(data=blob), blob
    eng.close()


def test_ffn_teacher_forced_logits(ffn_model):
    eng, ref, blob = ffn_model
    assert eng.cfg["no_feedforward"] == 0
    rng = np.random.default_rng(41)
    enc_ids = rng.integers(0, 8192, 200)
    dec_ids = np.r_[1, rng.integers(0, 8192, 7)]
    enc, lg = eng.debug_forward(enc_ids, dec_ids)
    renc, rlg = ref.forward(enc_ids, dec_ids)
    l_ex = np.abs(lg - rlg) - (ATOL + RTOL * np.abs(rlg))
    penc, _ = orc.Model(data=perturbed(blob, 4e-6, 7)).forward(enc_ids, dec_ids)
    sens = float(np.max(np.abs(penc - renc)))
    dev = float(np.max(np.abs(enc - renc)))
    print("logits max|d| %.3g (excess %.3g); encoder max|d| %.3g vs the oracle's own %.3g under 4e-6 noise" % (
        np.max(np.abs(lg - rlg)), l_ex.max(), dev, sens))
    assert l_ex.max() <= 0, l_ex.max()
    assert dev <= 3.0 * sens + ATOL, (dev, sens)


def test_ffn_batched_decode(ffn_model):
    eng, ref, _ = ffn_model
    ids, off = wl.random_prompts(192, 8, 60, 8192, seed=42)
    prompts = [ids[off[i]:off[i + 1]] for i in range(192)]
    steps = 4
    out, lens, lg = eng.run_batch_ids(prompts, steps, want_logits=True)
    tol = 2 * (ATOL + RTOL * 10.0)
    for r in (0, 91, 191):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, want_logits=True)
        assert close(lg[r, 0], rlg[0]), float(np.max(np.abs(lg[r, 0] - rlg[0])))
        for s in range(steps):  # the sequences may part only at a tie-level step
            if out[r, s] != rid[s]:
                assert rmarg[s] <= tol, (r, s)
                break
