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


def test_noalloc_attention_rejects_oversize_calls(pkg):
    L = pkg.lib()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    q, kv, ln = _inputs(7, 1, 16, 128, [128])
    out = torch.zeros((1, 16 * 64), dtype=torch.float32, device="cuda")
    # 64 rows x 16 heads x 65 splits of an 8196-position context exceeds the scratch
    rc = L.t3b_op_attention_noalloc(_p(q), _p(kv[0]), _p(kv[1]), 64, 16, 8196, _p(ln), _p(out), st)
    assert rc == -1
    assert "static scratch" in pkg.last_error()
