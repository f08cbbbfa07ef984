"""The allocation-free attention entry point (t3b_op_attention_noalloc).

It serves callers that may not allocate device memory while they decode:
hosts whose device memory is owned by their own pool allocator, and
real-time callers that cannot risk cudaMalloc's allocator locks or implicit
device synchronisation.  Its split-K scratch is a static device array, so
these tests check that two calls in a row (the second one reusing the
array's leftover contents) give exactly what the allocating entry point
t3b_op_attention gives, and that oversize calls are refused.

This file is named to be collected last: it must pass both alone in a fresh
process and after every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _p(t):
    return C.c_void_p(t.data_ptr())


def _inputs(seed, M, H, T, lens):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal((M, H * 64)).astype(np.float32)).cuda()
    kv = torch.from_numpy(np.stack([(rng.standard_normal((M, H, T, 64)) * 0.5).astype(np.float16),
                                    rng.standard_normal((M, H, T, 64)).astype(np.float16)])).cuda()
    ln = torch.from_numpy(np.asarray(lens, np.int32)).cuda()
    return q, kv, ln


def test_noalloc_attention_matches_allocating_entry_point_twice(pkg):
    L = pkg.lib()
    M, H, T = 3, 16, 2048
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, lens in enumerate(([2048, 300, 129], [1, 1500, 777])):
        q, kv, ln = _inputs(100 + call, M, H, T, lens)
        ref = torch.zeros((M, H * 64), dtype=torch.float32, device="cuda")
        got = torch.full((M, H * 64), float("nan"), dtype=torch.float32, device="cuda")
        pkg.check(L.t3b_op_attention(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(ln), _p(ref), st))
        pkg.check(L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(ln), _p(got), st))
        torch.cuda.synchronize()
        # same kernel, same inputs: identical up to float rounding (tolerance
        # kept at the attention tests' 1e-5 of max |out|)
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all()
        assert np.max(np.abs(g - r)) <= 1e-5 * np.max(np.abs(r)), call


def test_noalloc_attention_many_rows_matches_fp64(pkg):
    """From 8 query rows on both entry points run one CTA per (row, head)
    with no split scratch: the static array is not used and nothing bounds M
    but the counter limit.  Checked against the fp64 attention and against
    the allocating entry point, on two calls in a row."""
    L = pkg.lib()
    M, H, T = 9, 16, 1024
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        rng = np.random.default_rng(200 + call)
        lens = rng.integers(1, T + 1, M).astype(np.int32)
        q, kv, ln = _inputs(300 + call, M, H, T, lens)
        ref = torch.zeros((M, H * 64), dtype=torch.float32, device="cuda")
        got = torch.full((M, H * 64), float("nan"), dtype=torch.float32, device="cuda")
        pkg.check(L.t3b_op_attention(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(ln), _p(ref), st))
        pkg.check(L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(ln), _p(got), st))
        assert L.t3b_op_check(st) == 0
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.max(np.abs(g - r)) <= 1e-5 * np.max(np.abs(r)), call
        qn, kn, vn = q.cpu().numpy().astype(np.float64), kv[0].cpu().numpy(), kv[1].cpu().numpy()
        for m in range(M):
            for h in range(H):
                n = int(lens[m])
                s = (kn[m, h, :n].astype(np.float64) @ qn[m, h * 64:(h + 1) * 64]) / 8.0
                w = np.exp(s - s.max())
                o = (w[:, None] * vn[m, h, :n].astype(np.float64)).sum(0) / w.sum()
                assert np.max(np.abs(g[m, h * 64:(h + 1) * 64] - o)) <= 1e-5 * np.max(np.abs(o)), (call, m, h)


def test_noalloc_attention_length_error_is_kept_for_check(pkg):
    """A zero-length row is reported by t3b_op_check even after a later
    clean call: the error word is not cleared by the next call."""
    L = pkg.lib()
    M, H, T = 3, 16, 256
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    q, kv, _ = _inputs(9, M, H, T, [1, 1, 1])
    out = torch.zeros((M, H * 64), dtype=torch.float32, device="cuda")
    bad = torch.tensor([4, 0, 4], dtype=torch.int32, device="cuda")
    good = torch.tensor([4, 4, 4], dtype=torch.int32, device="cuda")
    pkg.check(L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(bad), _p(out), st))
    pkg.check(L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(good), _p(out), st))
    assert L.t3b_op_check(st) == -5
    assert L.t3b_op_check(st) == 0


def test_noalloc_attention_rejects_oversize_calls(pkg):
    L = pkg.lib()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    q, kv, ln = _inputs(7, 1, 16, 128, [128])
    out = torch.zeros((1, 16 * 64), dtype=torch.float32, device="cuda")
    # 7 rows (split-key kernel) x 40 heads x 65 splits of an 8196-position
    # context exceeds the partials; 64 rows x 65 heads exceeds the counters.
    # Both are refused before anything is launched.
    for M, H in ((7, 40), (64, 65)):
        rc = L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), M, H, 8196, _p(ln), _p(out), st)
        assert rc == -1
        assert "static scratch" in pkg.last_error()
