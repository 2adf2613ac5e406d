"""needle_ffn_forward_noalloc: the MLP block for callers that cannot allocate
device memory during a call (a fixed memory budget handed over at start-up,
latency-critical steps, embedders with their own memory manager).  Its
output must match needle_ffn_forward, through the C ABI, on two calls in a
row (the second call reuses the fixed array the first one wrote).  This file
is collected last so a failure here comes after every other test has run."""
import numpy as np
import pytest

from conftest import ATOL, RTOL, load_pkg

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

nb = load_pkg()
wl = load_pkg("needle_workload", "workload.py")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def dev(a):
    return torch.from_numpy(np.array(a, copy=True)).cuda()


def close_act(got, ref):
    # the activation tolerance of the parity tests: ATOL scaled by max(1, rms)
    atol = ATOL * max(1.0, float(np.sqrt(np.mean(np.square(ref, dtype=np.float64)))))
    return np.all(np.abs(got.astype(np.float64) - ref) <= atol + RTOL * np.abs(ref))


def run_both(T, act, seed):
    d, ff = 512, 2048
    rng = np.random.default_rng(seed)
    x = dev(rng.standard_normal((T, d)).astype(np.float32))
    w = [wl.random_int4(rng, d, ff), wl.random_int4(rng, d, ff), wl.random_int4(rng, ff, d)]
    wd = [[dev(a) for a in pair] for pair in w]
    ptrs = [[t.data_ptr() for t in pair] for pair in wd]
    ref = torch.full((T, d), float("nan"), device="cuda")
    got = torch.full((T, d), float("nan"), device="cuda")
    nb.ffn_forward(x.data_ptr(), T, d, ff, ptrs[0], ptrs[1], ptrs[2], act, ref.data_ptr())
    nb.ffn_forward_noalloc(x.data_ptr(), T, d, ff, ptrs[0], ptrs[1], ptrs[2], act, got.data_ptr())
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy().astype(np.float64)


def test_noalloc_matches_allocating_entry_point_twice():
    # two calls in a row with different inputs, sizes and activations
    for T, act, seed in ((256, 0, 1), (96, 1, 2)):
        got, ref = run_both(T, act, seed)
        assert not np.isnan(got).any()
        assert close_act(got, ref)


@pytest.mark.parametrize("T,act", [(1, 0), (1, 2), (8, 1), (8, 0)])
def test_noalloc_few_tokens(T, act):
    # up to 8 tokens the block runs on the matvec kernels (gate and up
    # interleaved, the activation in the epilogue)
    got, ref = run_both(T, act, 10 + T + act)
    assert not np.isnan(got).any()
    assert close_act(got, ref)


def test_noalloc_allocates_nothing():
    # The call must take nothing from the device's stream-ordered pool (the
    # allocator needle_ffn_forward uses): reset the pool's high-water mark,
    # call twice, and the mark must not have moved past the memory in use.
    rt = pytest.importorskip("cuda.bindings.runtime")
    drv = pytest.importorskip("cuda.bindings.driver")
    T, d, ff = 64, 512, 2048
    rng = np.random.default_rng(3)
    x = dev(rng.standard_normal((T, d)).astype(np.float32))
    w = [[dev(a) for a in wl.random_int4(rng, d if i < 2 else ff, ff if i < 2 else d)] for i in range(3)]
    ptrs = [[t.data_ptr() for t in pair] for pair in w]
    out = torch.empty((T, d), device="cuda")
    nb.ffn_forward_noalloc(x.data_ptr(), T, d, ff, ptrs[0], ptrs[1], ptrs[2], 0, out.data_ptr())
    torch.cuda.synchronize()
    err, pool = rt.cudaDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == rt.cudaError_t.cudaSuccess
    used_high = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh
    used_now = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent
    (err,) = rt.cudaMemPoolSetAttribute(pool, used_high, drv.cuuint64_t(0))  # 0 resets the mark to current use
    assert err == rt.cudaError_t.cudaSuccess
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        nb.ffn_forward_noalloc(x.data_ptr(), T, d, ff, ptrs[0], ptrs[1], ptrs[2], 0, out.data_ptr())
    torch.cuda.synchronize()
    err, high = rt.cudaMemPoolGetAttribute(pool, used_high)
    err2, now = rt.cudaMemPoolGetAttribute(pool, used_now)
    assert err == err2 == rt.cudaError_t.cudaSuccess
    assert int(high) == int(now)
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_oversize():
    x = torch.zeros(1, device="cuda")
    p = x.data_ptr()
    with pytest.raises(nb.NeedleError, match="exceeds the fixed hidden buffer"):
        nb.ffn_forward_noalloc(p, 513, 512, 2048, [p, p], [p, p], [p, p], 0, p)
    # few tokens over a wide hidden layer: the shared-memory limit, named
    with pytest.raises(nb.NeedleError, match="shared memory"):
        nb.ffn_forward_noalloc(p, 8, 512, 8192, [p, p], [p, p], [p, p], 0, p)
