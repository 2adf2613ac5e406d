"""needle_run / needle_run_stream / needle_run_batch on the GPU against
run_impl (crates/needle-infer/src/engine.rs:226-322) restated on the oracle:
the Python front end (oracle/text_oracle.py) builds the encoder input and the
constrained-decoding state, the C++ oracle model gives the logits of each
step (teacher-forced forward over the tokens so far), the mask is added as
the reference adds it and the last maximal index is taken.  Random-init model
at the shipped dims with max_dec_len 12 (every oracle step re-runs the
forward), synthetic SentencePiece vocabulary of 8192 pieces.  Token ids must
match up to the first step whose oracle top-2 margin is within the logit
tolerance; with no such step the output text must match exactly.

The step-wise batch API that the text path drives is checked separately:
masks set step by step through needle_batch_set_step_mask give the tokens
of the same masks passed up front to needle_run_batch_ids."""
import numpy as np
import pytest

import oracle as orc
import text_oracle as to
from conftest import ATOL, RTOL, load_pkg

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")
STEPS = 12
VOCAB = wl.random_vocab(8192, 0)
TOL = 2 * (ATOL + RTOL * 10.0)

CASES = [
    ("What's the weather in Paris?", '[{"name":"getWeather","parameters":{"city":{"type":"string"}}}]'),
    ("Please book a flight from New York", '[ {"name": "bookFlight", "parameters": {"from": {}, "to": {}}} ]'),
    ("Search for Python tutorials online", "[]"),
    ("naïve café 中文 🙂", '[{"name":"HTMLParser","parameters":{"type":"object","properties":{"url":{}}}}]'),
    ("x " * 1100, '[{"name":"t","parameters":{}}]'),  # longer than max_enc_len: truncated
    ("", '[{"name":"only_tools","parameters":{"a":{}}}]'),
]


@pytest.fixture(scope="module")
def models():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    blob = wl.random_model(seed=21, max_dec_len=STEPS, contrastive=(256, 128))
    return nb.NeedleEngine.from_bytes(blob, VOCAB), orc.Model(data=blob), to.Vocab(VOCAB)


def reference_run(model, vocab, query, tools, V, max_enc):
    enc, defs = to.encoder_input(vocab, query, tools, max_enc)
    if not enc:
        return [], [], ""
    cd = to.ConstrainedDecoder(defs, vocab)
    dec, out, margins = [to.EOS], [], []
    for _ in range(STEPS):
        lg = model.forward(enc, dec)[1][-1].astype(np.float32)
        ok = cd.allowed(V)
        if ok is not None:
            m = np.full(V, np.float32(-1e9), np.float32)
            m[ok] = 0.0
            lg = lg + m
        best = int(np.flatnonzero(lg == lg.max())[-1])
        rest = np.delete(lg, best)
        margins.append(float(lg[best] - rest.max()))
        if best == to.EOS:
            break
        out.append(best)
        dec.append(best)
        cd.update(best)
    raw = vocab.decode_ids(out)
    tc = vocab.piece_text(to.TOOL_CALL)
    if tc and raw.startswith(tc):
        raw = raw[len(tc):]
    return out, margins, to.restore_tool_names(raw, defs)


@pytest.mark.parametrize("case", range(len(CASES)))
def test_run_matches_reference(models, case):
    eng, model, vocab = models
    query, tools = CASES[case]
    streamed = []
    text = eng.run_stream(query, tools, lambda tid, piece: streamed.append((tid, piece)))
    assert eng.run(query, tools) == text
    ref_ids, margins, ref_text = reference_run(model, vocab, query, tools, eng.cfg["vocab_size"],
                                               eng.cfg["max_enc_len"])
    got = [t for t, _ in streamed]
    assert all(p == vocab.piece_text(t) for t, p in streamed)
    for s in range(len(margins)):
        # a stopped run emitted EOS at this step
        r = ref_ids[s] if s < len(ref_ids) else to.EOS
        g = got[s] if s < len(got) else to.EOS
        if g != r:
            assert margins[s] <= TOL, (s, got, ref_ids)
            return  # a near-tie: the sequences may legitimately part here
    assert len(got) == len(ref_ids)
    assert text == ref_text


def test_run_batch_matches_single_runs(models):
    eng, _, _ = models
    qs = [c[0] for c in CASES]
    ts = [c[1] for c in CASES]
    assert eng.run_batch(qs, ts) == [eng.run(q, t) for q, t in zip(qs, ts)]


def test_run_empty_and_bad_input(models):
    eng, _, _ = models
    assert eng.run("", "") == ""  # the reference returns early on an empty encoder input
    L = nb.lib()
    assert not L.needle_run(eng._h, b"\xff", b"[]")
    assert not L.needle_run(None, b"q", b"[]")


def test_step_masks_match_upfront_masks(models):
    eng, _, _ = models
    V = eng.cfg["vocab_size"]
    ids, off = wl.random_prompts(5, 8, 40, V, seed=31)
    masks = wl.random_masks(5, STEPS, V, 0.05, seed=32)
    ref_ids, ref_lens = eng.run_batch_ids([ids[off[i]:off[i + 1]] for i in range(5)], STEPS, mask_bits=masks,
                                          stop_on_eos=True)
    ones = np.full_like(masks, np.uint64(0xFFFFFFFFFFFFFFFF))
    b = eng.prepare_batch(ids, off, STEPS, ones, flags=nb.STOP_ON_EOS)
    try:
        b.begin()
        done = np.zeros(5, bool)
        for s in range(STEPS):
            b.set_step_mask(s, masks[:, s, :])
            tok, lens, d = b.step()
            for r in range(5):
                if not done[r] and not d[r]:
                    assert tok[r] == ref_ids[r, s], (r, s)
            done |= d.astype(bool)
        assert np.array_equal(lens, ref_lens)
    finally:
        b.close()


# ── contrastive head (engine.rs:24-217) ───────────────────────────────────

DESCS = ["Get the current weather for a city", "Send an email message", "Book a flight between two cities",
         "", "Search the web", "Set an alarm for a time", "naïve café 中文"]


def test_encode_contrastive_matches_reference(models):
    eng, model, vocab = models
    assert eng.contrastive_dim == model.contrastive_dim == 128
    for text in ["What's the weather in Paris?"] + DESCS:
        got = eng.encode_contrastive(text)
        ref = model.encode_contrastive(vocab.encode(text))
        assert np.all(np.abs(got - ref) <= ATOL + RTOL * np.abs(ref)), (text, float(np.max(np.abs(got - ref))))
    assert not np.any(eng.encode_contrastive("   "))  # no tokens: the zero vector


def test_retrieve_tools_matches_reference(models):
    eng, model, vocab = models
    query = "What's the weather in Paris?"
    got = eng.retrieve_tools(query, DESCS, 4)
    q = model.encode_contrastive(vocab.encode(query))
    ref = [float(np.dot(q, model.encode_contrastive(vocab.encode(t)))) for t in DESCS]
    order = sorted(range(len(DESCS)), key=lambda i: -ref[i])  # stable: ties keep index order
    assert len(got) == 4
    for r, (i, sc) in enumerate(got):
        assert abs(sc - ref[i]) <= 1e-4
        if r + 1 < len(DESCS) and abs(ref[order[r]] - ref[order[r + 1]]) > 1e-3:
            assert i == order[r]
    assert eng.retrieve_tools(query, DESCS, 100)[-1][0] in range(len(DESCS))
    assert eng.retrieve_tools(query, [], 3) == []


def test_no_contrastive_head():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    eng = nb.NeedleEngine.from_bytes(wl.random_model(seed=22, num_encoder_layers=1, num_decoder_layers=1), VOCAB)
    try:
        assert eng.contrastive_dim == 0 and eng.encode_contrastive("x") is None
        assert eng.retrieve_tools("x", ["a", "b"], 2) == []
    finally:
        eng.close()
