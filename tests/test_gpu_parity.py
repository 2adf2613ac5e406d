"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Tolerances: INT4 packing / unpacking bit-exact; logits |gpu - ref| <= ATOL +
RTOL * |ref| with RTOL = 1e-3, ATOL = 1e-4; intermediate activations (encoder
hidden, matmul and MLP outputs) the same with ATOL scaled by the tensor's RMS
when that exceeds 1 (f32 rounding error grows with the magnitude of the sum,
not of each element); greedy and constrained token ids identical wherever the
oracle's top-2 margin exceeds the logit tolerance (the sequences may part
only at a tie-level step, and legitimately differ after it).
"""
import json
import os

import numpy as np
import pytest

import oracle as orc
from conftest import ATOL, GOLDEN, RTOL, load_pkg

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")
V_TINY = json.load(open(os.path.join(GOLDEN, "tiny_vectors.json")))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def close(got, ref):
    """Logit tolerance."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.all(np.abs(got - ref) <= ATOL + RTOL * np.abs(ref))


def max_excess(got, ref, scaled=False):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    atol = ATOL * max(1.0, float(np.sqrt(np.mean(ref * ref)))) if scaled else ATOL
    return float(np.max(np.abs(got - ref) - (atol + RTOL * np.abs(ref))))


def close_act(got, ref):
    """Activation tolerance: ATOL scaled by max(1, rms(ref))."""
    return max_excess(got, ref, scaled=True) <= 0.0


def tokens_match(gpu_ids, ref_ids, ref_margins, tol_margin):
    """Exact match, except that the sequences may part at a step whose
    oracle top-2 margin is within the logit tolerance (a tie the tolerance
    cannot resolve); after that step they legitimately differ."""
    for s, (g, r) in enumerate(zip(gpu_ids, ref_ids)):
        if g != r:
            return ref_margins[s] <= tol_margin
    return True


# ── INT4 kernels ────────────────────────────────────────────────────────────

@pytest.mark.parametrize("M,N,K", [(1, 2048, 512), (1, 512, 512), (3, 256, 512), (8, 512, 2048), (1, 8192, 512),
                                   (9, 512, 512), (64, 512, 512), (200, 2048, 512), (512, 512, 2048),
                                   (1, 8, 33), (5, 16, 65), (130, 24, 33), (17, 40, 96), (2, 6, 16)])
def test_int4_matmul_vs_oracle(M, N, K):
    x, packed, scales = wl.int4_case(M, N, K, seed=M * 7 + N + K)
    ref = orc.matmul(packed, scales, K, N, x, path=1)
    xd, wd, sd = dev(x), dev(packed), dev(scales)
    y = torch.full((M, N), float("nan"), device="cuda")
    nb.int4_matmul(xd.data_ptr(), M, K, wd.data_ptr(), sd.data_ptr(), N, scales.shape[0], y.data_ptr())
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert not np.isnan(got).any()
    assert close_act(got, ref), max_excess(got, ref, True)


@pytest.mark.parametrize("M", [1, 2, 5, 8])
def test_int4_matmul_overlap_chain(M):
    """Launches with programmatic dependent launch, each reading the previous
    launch's output as its x: the weight prefetch overlaps, the x read waits."""
    d, steps = 512, 6
    cases = [wl.int4_case(M, d, d, seed=100 + i) for i in range(steps)]
    x0 = cases[0][0]
    bufs = [dev(x0)] + [torch.full((M, d), float("nan"), device="cuda") for _ in range(steps)]
    ws = [(dev(c[1]), dev(c[2])) for c in cases]
    for i in range(steps):
        nb.int4_matmul(bufs[i].data_ptr(), M, d, ws[i][0].data_ptr(), ws[i][1].data_ptr(), d, cases[i][2].shape[0],
                       bufs[i + 1].data_ptr(), overlap=True)
    torch.cuda.synchronize()
    for i in range(steps):
        xin = bufs[i].cpu().numpy()
        ref = orc.matmul(cases[i][1], cases[i][2], d, d, xin, path=1)
        got = bufs[i + 1].cpu().numpy()
        assert not np.isnan(got).any(), i
        assert close_act(got, ref), (i, max_excess(got, ref, True))


@pytest.mark.parametrize("M", [1, 8, 127, 128, 200, 512])
def test_int4_plan_vs_oracle(M):
    N, K = 2048, 512
    x, packed, scales = wl.int4_case(M, N, K, seed=3 * M + 1)
    ref = orc.matmul(packed, scales, K, N, x, path=1)
    wd, sd = dev(packed), dev(scales)
    plan = nb.Int4Plan(wd.data_ptr(), sd.data_ptr(), K, N, scales.shape[0], max_m=512)
    try:
        xd = dev(x)
        for rep in range(2):  # the workspace is reused across calls
            y = torch.full((M, N), float("nan"), device="cuda")
            plan.matmul(xd.data_ptr(), M, y.data_ptr(), overlap=(rep == 1))
            plan.status()
            got = y.cpu().numpy()
            assert not np.isnan(got).any()
            assert close_act(got, ref), max_excess(got, ref, True)
        with pytest.raises(nb.NeedleError):
            plan.matmul(xd.data_ptr(), 513, y.data_ptr())
    finally:
        plan.close()


@pytest.mark.parametrize("M,max_m,N,K", [(9, 64, 512, 512), (64, 64, 512, 2048), (33, 40, 8192, 512)])
def test_int4_plan_short_workspace_vs_oracle(M, max_m, N, K):
    # plans for fewer than 128 rows still take the tensor-core GEMM from 9
    # rows: x is staged in a one-tile (128-row) workspace whose extra rows are
    # never stored
    x, packed, scales = wl.int4_case(M, N, K, seed=5 * M + N)
    ref = orc.matmul(packed, scales, K, N, x, path=1)
    wd, sd = dev(packed), dev(scales)
    plan = nb.Int4Plan(wd.data_ptr(), sd.data_ptr(), K, N, scales.shape[0], max_m=max_m)
    try:
        y = torch.full((M, N), float("nan"), device="cuda")
        plan.matmul(dev(x).data_ptr(), M, y.data_ptr())
        plan.status()
        got = y.cpu().numpy()
        assert not np.isnan(got).any()
        assert close_act(got, ref), max_excess(got, ref, True)
    finally:
        plan.close()


@pytest.mark.parametrize("M,N,K", [(4800, 2176, 512), (4736, 2048, 96)])
def test_int4_plan_wide_tiles_vs_oracle(M, N, K):
    # Tall matrices take the 128 x 256 output tiles; N = 2176 leaves a
    # half-empty last column tile, M = 4800 a partial last row tile.
    x, packed, scales = wl.int4_case(M, N, K, seed=M + N)
    rows = np.r_[0:64, M // 2 - 32:M // 2 + 32, M - 64:M]
    ref = orc.matmul(packed, scales, K, N, x[rows], path=1)
    wd, sd = dev(packed), dev(scales)
    plan = nb.Int4Plan(wd.data_ptr(), sd.data_ptr(), K, N, scales.shape[0], max_m=M)
    try:
        y = torch.full((M, N), float("nan"), device="cuda")
        plan.matmul(dev(x).data_ptr(), M, y.data_ptr())
        plan.status()
        got = y.cpu().numpy()
        assert not np.isnan(got).any()
        assert close_act(got[rows], ref), max_excess(got[rows], ref, True)
    finally:
        plan.close()


@pytest.mark.parametrize("K,N", [(512, 2048), (33, 8), (65, 16), (16, 8), (4, 4), (2048, 24), (96, 40)])
def test_int4_quantize_bit_exact(K, N):
    rng = np.random.default_rng(K * N)
    w = (rng.standard_normal((K, N)) * 0.7).astype(np.float32)
    w[0, 0] = 0.0
    w[1, :] *= 50.0
    data, scales = orc.quantize(w)
    dd = torch.zeros(data.size, dtype=torch.uint8, device="cuda")
    ds = torch.zeros(scales.shape, dtype=torch.float32, device="cuda")
    nb.int4_quantize(dev(w).data_ptr(), K, N, dd.data_ptr(), ds.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(dd.cpu().numpy(), data)
    assert np.array_equal(ds.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    out = torch.zeros((K, N), dtype=torch.float32, device="cuda")
    nb.int4_dequantize(dd.data_ptr(), ds.data_ptr(), K, N, scales.shape[0], out.data_ptr())
    torch.cuda.synchronize()
    ref = orc.dequantize(data, scales, K, N)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_int4_quantize_golden_kat():
    kat = json.load(open(os.path.join(GOLDEN, "packing_kat.json")))
    for c in kat["cases"]:
        K, N = c["in_feat"], c["out_feat"]
        w = np.frombuffer(bytes.fromhex(c["w_f32_hex"]), np.float32).reshape(K, N)
        db, ng = orc.quant_sizes(K, N)
        dd = torch.zeros(db, dtype=torch.uint8, device="cuda")
        ds = torch.zeros(ng * N, dtype=torch.float32, device="cuda")
        nb.int4_quantize(dev(w).data_ptr(), K, N, dd.data_ptr(), ds.data_ptr())
        torch.cuda.synchronize()
        assert dd.cpu().numpy().tobytes().hex() == c["packed_hex"]
        assert ds.cpu().numpy().tobytes().hex() == c["scales_f32_hex"]


def test_int4_quantize_ties_round_away():
    w = np.zeros((32, 1), np.float32)
    w[:6, 0] = [7.0, 0.5, 1.5, 2.5, -0.5, -2.5]
    data, scales = orc.quantize(w)
    dd = torch.zeros(data.size, dtype=torch.uint8, device="cuda")
    ds = torch.zeros(1, dtype=torch.float32, device="cuda")
    nb.int4_quantize(dev(w).data_ptr(), 32, 1, dd.data_ptr(), ds.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(dd.cpu().numpy(), data)


@pytest.mark.parametrize("act,T", [(0, 64), (1, 64), (2, 64), (0, 256), (1, 200)])
def test_ffn_forward_vs_oracle(act, T):
    # ffn.rs:19-56 over T tokens (the MLP block), d=512 -> 2048 -> 512;
    # T >= 128 runs the tensor-core GEMM.
    d, ff = 512, 2048
    rng = np.random.default_rng(act + T)
    x = rng.standard_normal((T, d)).astype(np.float32)
    g, u, dn = wl.random_int4(rng, d, ff), wl.random_int4(rng, d, ff), wl.random_int4(rng, ff, d)
    ref = np.stack([orc.ffn_forward(g, u, dn, d, ff, x[t], act) for t in range(T)])
    gd = [dev(a) for a in g]
    ud = [dev(a) for a in u]
    dd = [dev(a) for a in dn]
    out = torch.full((T, d), float("nan"), device="cuda")
    nb.ffn_forward(dev(x).data_ptr(), T, d, ff, [t.data_ptr() for t in gd], [t.data_ptr() for t in ud],
                   [t.data_ptr() for t in dd], act, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert close_act(got, ref), max_excess(got, ref, True)


# ── tiny golden model (tests/vectors.json of the reference) ────────────────

@pytest.fixture(scope="module")
def tiny():
    blob = open(os.path.join(GOLDEN, "tiny_model.safetensors"), "rb").read()
    return nb.NeedleEngine.from_bytes(blob, "<pad>\n</s>\n"), orc.Model(data=blob)


def test_tiny_forward_golden(tiny):
    eng, ref = tiny
    enc_ids, start = V_TINY["inputs"]["enc_ids"], V_TINY["inputs"]["dec_start_id"]
    enc, lg = eng.debug_forward(enc_ids, [start])
    # the reference's own tolerances (parity_tests.rs:442-528)
    assert np.max(np.abs(lg[0] - np.array(V_TINY["forward"]["logits_q"]))) < 0.05
    assert np.max(np.abs(enc.ravel() - np.array(V_TINY["forward"]["enc_out_q"]).ravel())) < 0.05
    assert int(np.argmax(lg[0])) == V_TINY["forward"]["pred_token_q"]
    renc, rlg = ref.forward(enc_ids, [start])
    assert close(lg, rlg), max_excess(lg, rlg)
    assert close_act(enc, renc), max_excess(enc, renc, True)


def test_tiny_multi_step_golden(tiny):
    eng, ref = tiny
    steps = V_TINY["multi_step"]["steps"]
    ids, lens = eng.run_batch_ids([V_TINY["inputs"]["enc_ids"]], len(steps))
    for g, st in zip(ids[0], steps):
        if st["margin"] > 0.05:
            assert g == st["pred_token"]
        else:
            assert g in st["top5_tokens"]


# ── full-size random-init model (shipped config dims) ──────────────────────

@pytest.fixture(scope="module")
def full():
    blob = wl.random_model(seed=11)
    return nb.NeedleEngine.from_bytes(blob, "a\nb\n"), orc.Model(data=blob)


def test_full_teacher_forced_logits(full):
    eng, ref = full
    rng = np.random.default_rng(5)
    enc_ids = rng.integers(0, 8192, 256)
    dec_ids = np.concatenate([[1], rng.integers(0, 8192, 7)])
    renc, rlg = ref.forward(enc_ids, dec_ids)
    enc, lg = eng.debug_forward(enc_ids, dec_ids)
    print("teacher-forced: enc max|d| %.3g, logits max|d| %.3g, logit excess %.3g" % (
        np.max(np.abs(enc - renc)), np.max(np.abs(lg - rlg)), max_excess(lg, rlg)))
    assert close_act(enc, renc), max_excess(enc, renc, True)
    assert close(lg, rlg), max_excess(lg, rlg)


def test_full_greedy_64_steps(full):
    # The single-request workload: a 256-token prompt, 64 greedy steps, no mask.
    eng, ref = full
    rng = np.random.default_rng(6)
    enc_ids = rng.integers(0, 8192, 256)
    rid, rmarg = ref.generate(enc_ids, 64)
    ids, lens = eng.run_batch_ids([enc_ids], 64)
    assert lens[0] == 64
    tol = 2 * (ATOL + RTOL * 10.0)
    assert tokens_match(ids[0], rid, rmarg, tol)


def test_full_batch_masked_vs_oracle(full):
    # Constrained batched decode: ragged prompts incl. the extremes 1 and
    # max_enc_len, 5% random masks with one forced token per step.
    eng, ref = full
    lens_in = [1, 64, 300, 1024, 17, 512]
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 8192, n) for n in lens_in]
    steps = 6
    masks = wl.random_masks(len(prompts), steps, 8192, 0.05, seed=8)
    ids, lens, lg = eng.run_batch_ids(prompts, steps, mask_bits=masks, want_logits=True)
    tol = 2 * (ATOL + RTOL * 10.0)
    for r, p in enumerate(prompts):
        rid, rmarg, rlg = ref.generate(p, steps, mask_bits=masks[r], want_logits=True)
        assert tokens_match(ids[r], rid, rmarg, tol), r
        allowed = np.unpackbits(masks[r].view(np.uint8), axis=-1, bitorder="little")[:, :8192].astype(bool)
        for s in range(steps):
            assert allowed[s, ids[r, s]]
            if ids[r, :s].tolist() != rid[:s].tolist():
                break
            assert close(lg[r, s], rlg[s]), (r, s, max_excess(lg[r, s], rlg[s]))


def test_eos_stops_request(full):
    # engine.rs:306-308: EOS ends generation and is not emitted.
    eng, ref = full
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 8192, 40), rng.integers(0, 8192, 90)]
    steps = 12
    masks = np.full((2, steps, 128), np.uint64(0xFFFFFFFFFFFFFFFF))
    masks[0, 4] = 0
    masks[0, 4, 0] = np.uint64(1 << 1)  # step 4 of request 0 may only emit EOS
    ids, lens = eng.run_batch_ids(prompts, steps, mask_bits=masks, stop_on_eos=True)
    rid, _ = ref.generate(prompts[0], steps, mask_bits=masks[0], stop_on_eos=True)
    assert lens[0] == 4 == len(rid)
    assert lens[1] == steps
    assert ids[0, :4].tolist() == rid.tolist()


def test_batch_rows_are_independent(full):
    eng, _ = full
    ids_in, off = wl.random_prompts(40, 8, 200, 8192, seed=10)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(40)]
    all_ids, _, all_lg = eng.run_batch_ids(prompts, 4, want_logits=True)
    for r in (0, 17, 39):
        one, _, lg = eng.run_batch_ids([prompts[r]], 4, want_logits=True)
        assert close(all_lg[r, 0], lg[0, 0])


def test_batched_decode_tensor_core_vs_oracle(full):
    # 160 requests: the decode projections run as 160-row tensor-core GEMMs.
    eng, ref = full
    ids_in, off = wl.random_prompts(160, 8, 96, 8192, seed=12)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(160)]
    steps = 5
    masks = wl.random_masks(160, steps, 8192, 0.05, seed=13)
    ids, lens, lg = eng.run_batch_ids(prompts, steps, mask_bits=masks, want_logits=True)
    tol = 2 * (ATOL + RTOL * 10.0)
    for r in (0, 1, 77, 159):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, mask_bits=masks[r], want_logits=True)
        assert tokens_match(ids[r], rid, rmarg, tol), r
        assert close(lg[r, 0], rlg[0]), max_excess(lg[r, 0], rlg[0])


def test_long_decode_vs_oracle(full):
    # 72 greedy steps: the decoder self-attention passes over more than 64
    # cached positions, on the 136-request path (attention output written as
    # the output projection's operand planes) and on the single-request path.
    eng, ref = full
    ids_in, off = wl.random_prompts(136, 8, 40, 8192, seed=15)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(136)]
    steps = 72
    ids, lens, lg = eng.run_batch_ids(prompts, steps, want_logits=True)
    one, _, lg1 = eng.run_batch_ids([prompts[3]], steps, want_logits=True)
    tol = 2 * (ATOL + RTOL * 10.0)
    for r, got, glg in ((0, ids[0], lg[0]), (3, ids[3], lg[3]), (135, ids[135], lg[135]), (3, one[0], lg1[0])):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, want_logits=True)
        assert tokens_match(got, rid, rmarg, tol), r
        for s in range(steps):
            if got[:s].tolist() != rid[:s].tolist():
                break
            assert close(glg[s], rlg[s]), (r, s, max_excess(glg[s], rlg[s]))


def test_pdl_and_graphs_change_nothing(full):
    # Programmatic dependent launch and the step graphs only change when
    # kernels start: tokens and logits are bit-identical with and without
    # them (20 steps: the self-attention pass sizes 16 and 32 both run).
    eng, _ = full
    ids_in, off = wl.random_prompts(144, 8, 80, 8192, seed=16)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(144)]
    masks = wl.random_masks(144, 20, 8192, 0.05, seed=17)
    ref = eng.run_batch_ids(prompts, 20, mask_bits=masks, want_logits=True, graph=False, pdl=False)
    for graph, pdl in ((True, True), (False, True), (True, False)):
        got = eng.run_batch_ids(prompts, 20, mask_bits=masks, want_logits=True, graph=graph, pdl=pdl)
        assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1]), (graph, pdl)
        assert np.array_equal(got[2], ref[2]), (graph, pdl)


def test_multi_chunk_prefill_vs_oracle(full):
    # Over 524,288 prompt tokens, so the prefill runs in two chunks: requests
    # on both sides of the chunk boundary, and the first and last, match the
    # oracle.
    eng, ref = full
    n = 1100
    ids_in, off = wl.random_prompts(n, 490, 512, 8192, seed=18)
    assert int(off[-1]) > 524288
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(n)]
    steps = 2
    ids, lens, lg = eng.run_batch_ids(prompts, steps, want_logits=True)
    first2 = int(np.searchsorted(off, 524288, side="right")) - 1  # the request that opens chunk 2
    tol = 2 * (ATOL + RTOL * 10.0)
    for r in (0, first2 - 1, first2, n - 1):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, want_logits=True)
        assert tokens_match(ids[r], rid, rmarg, tol), r
        assert close(lg[r, 0], rlg[0]), (r, max_excess(lg[r, 0], rlg[0]))


def test_wide_prefill_tiles_vs_oracle(full):
    # Over 9,500 prompt rows: every prefill projection (the fused QKV with its
    # norm + RoPE epilogue included) runs with 128 x 256 output tiles.
    eng, ref = full
    ids_in, off = wl.random_prompts(96, 100, 128, 8192, seed=14)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(96)]
    steps = 3
    ids, lens, lg = eng.run_batch_ids(prompts, steps, want_logits=True)
    tol = 2 * (ATOL + RTOL * 10.0)
    for r in (0, 50, 95):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, want_logits=True)
        assert tokens_match(ids[r], rid, rmarg, tol), r
        assert close(lg[r, 0], rlg[0]), max_excess(lg[r, 0], rlg[0])


def test_argument_errors(full):
    eng, _ = full
    with pytest.raises(nb.NeedleError, match="out of range"):
        eng.run_batch_ids([[8192]], 2)
    with pytest.raises(nb.NeedleError, match="max_dec_len"):
        eng.run_batch_ids([[5]], 513)
    with pytest.raises(nb.NeedleError, match="prompt tokens"):
        eng.run_batch_ids([list(range(1025))], 2)
    ids, lens = eng.run_batch_ids([[3, 4]], 0)
    assert lens[0] == 0


@pytest.mark.parametrize("act,T", [(0, 256), (1, 64), (2, 200), (0, 5), (1, 1)])
def test_ffn_plan_vs_oracle(act, T):
    # The prepared MLP block: the gate|up GEMM's epilogue writes the hidden
    # activation as the down GEMM's operand planes (tensor cores from 9
    # tokens), the CUDA-core kernels below; two calls in a row reuse the
    # plan's workspace.
    d, ff = 512, 2048
    rng = np.random.default_rng(40 + act + T)
    x = rng.standard_normal((T, d)).astype(np.float32)
    g, u, dn = wl.random_int4(rng, d, ff), wl.random_int4(rng, d, ff), wl.random_int4(rng, ff, d)
    ref = np.stack([orc.ffn_forward(g, u, dn, d, ff, x[t], act) for t in range(T)])
    gd, ud, dd = [dev(a) for a in g], [dev(a) for a in u], [dev(a) for a in dn]
    plan = nb.FfnPlan(d, ff, [t.data_ptr() for t in gd], [t.data_ptr() for t in ud], [t.data_ptr() for t in dd],
                      max_t=256)
    try:
        xd = dev(x)
        for _ in range(2):
            out = torch.full((T, d), float("nan"), device="cuda")
            plan.forward(xd.data_ptr(), T, act, out.data_ptr())
            plan.status()
            got = out.cpu().numpy()
            assert close_act(got, ref), max_excess(got, ref, True)
        with pytest.raises(nb.NeedleError):
            plan.forward(xd.data_ptr(), 257, act, out.data_ptr())
    finally:
        plan.close()


def test_one_row_tile_batch_vs_oracle(full):
    # 128 requests: every decode GEMM has a single 128-row tile, so the
    # projections and the head's mask + argmax epilogue run as split-K
    # clusters reduced through distributed shared memory.
    eng, ref = full
    ids_in, off = wl.random_prompts(128, 8, 70, 8192, seed=19)
    prompts = [ids_in[off[i]:off[i + 1]] for i in range(128)]
    steps = 4
    masks = wl.random_masks(128, steps, 8192, 0.05, seed=20)
    ids, lens, lg = eng.run_batch_ids(prompts, steps, mask_bits=masks, want_logits=True)
    again = eng.run_batch_ids(prompts, steps, mask_bits=masks, want_logits=True)
    assert np.array_equal(again[2], lg)  # the split-K reduction order is fixed
    tol = 2 * (ATOL + RTOL * 10.0)
    for r in (0, 64, 127):
        rid, rmarg, rlg = ref.generate(prompts[r], steps, mask_bits=masks[r], want_logits=True)
        assert tokens_match(ids[r], rid, rmarg, tol), r
        assert close(lg[r, 0], rlg[0]), max_excess(lg[r, 0], rlg[0])
