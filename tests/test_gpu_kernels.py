"""GPU parity tests of the individual kernels, called through the C ABI
(t3b_op_*), against the CPU oracle on the same seeded inputs."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err, synth_logits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def test_device_exp_equals_host_libm_expf_exhaustive(pkg, orc):
    """Every float in [-104, 0] (the arguments the sampler's exp can see):
    device exp == the host C library's expf, bit for bit."""
    L = pkg.lib()
    orc.set_threads(8)
    lo = 0x80000000
    hi = int(np.array([-104.0], np.float32).view(np.uint32)[0])
    chunk = 1 << 26
    bad = 0
    for a in range(lo, hi + 1, chunk):
        b = min(hi + 1, a + chunk)
        bits = np.arange(a, b, dtype=np.uint64).astype(np.uint32)
        x = bits.view(np.float32)
        ref = orc.expf_batch(x)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        pkg.check(L.t3b_op_expf(_p(xd), _p(yd), x.size, _stream()))
        y = yd.cpu().numpy()
        bad += int(np.count_nonzero(y.view(np.uint32) != ref.view(np.uint32)))
    x0 = np.array([0.0], np.float32)
    xd = torch.from_numpy(x0).cuda(); yd = torch.empty_like(xd)
    pkg.check(L.t3b_op_expf(_p(xd), _p(yd), 1, _stream()))
    assert float(yd.cpu()[0]) == 1.0
    assert bad == 0


def _quantized(ty, N, K, seed):
    import gguf
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    if ty == 1:
        return w.astype(np.float16)
    qt = {2: gguf.GGMLQuantizationType.Q4_0, 8: gguf.GGMLQuantizationType.Q8_0}[ty]
    return np.ascontiguousarray(gguf.quants.quantize(w, qt))


@pytest.mark.parametrize("ty", [2, 8, 1])
@pytest.mark.parametrize("KN", [(1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)])
@pytest.mark.parametrize("M", [1, 2, 8, 19, 32, 128])
def test_gemv_matches_oracle(pkg, orc, ty, KN, M):
    K, N = KN
    L = pkg.lib()
    q = _quantized(ty, N, K, seed=K + N + ty)
    rb = L.t3b_op_row_bytes(ty, K)
    wd = torch.empty(N * rb, dtype=torch.uint8, device="cuda")
    pkg.check(L.t3b_op_repack(ty, q.ctypes.data, N, K, _p(wd)))
    rng = np.random.default_rng(M * 7 + ty)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(K)).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    for epi, ln in ((0, False), (1, True), (2, False)):
        yd = torch.from_numpy(res.copy()).cuda()
        gd, bd = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
        biasd = torch.from_numpy(bias).cuda()
        pkg.check(L.t3b_op_gemv(ty, _p(wd), N, K, _p(xd), M, _p(gd) if ln else None, _p(bd) if ln else None,
                                1e-5, _p(biasd), _p(yd) if epi == 2 else None, epi, _p(yd), _stream()))
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        xin = x.copy()
        if ln:
            for m in range(M):
                orc.lib().orc_layernorm(np.ascontiguousarray(x[m]), K, g, b, 1e-5, xin[m])
        ref = np.zeros((M, N), np.float32)
        orc.lib().orc_matvec(ty, q.ctypes.data, N, K, np.ascontiguousarray(xin), M, bias.ctypes.data, ref, 1)
        if epi == 1:
            ref = np.vectorize(lambda v: orc.lib().orc_gelu(float(v), 1), otypes=[np.float32])(ref)
        if epi == 2:
            ref = ref + res
        # the GELU epilogue rounds through f16: an input 1 ulp away from the
        # oracle's can land on the neighbouring f16 (2^-11 relative)
        tol = 1e-3 if epi == 1 else 2e-4
        assert rel_err(y, ref) < tol, (ty, K, N, M, epi)
        if ty != 1 and M >= 5 and epi == 0:
            # the tensor-core GEMM (M >= 5) adds the per-block terms in block
            # order, as the oracle's restatement of ggml's dot does: identical
            assert np.array_equal(y, ref), (ty, K, N, M, float(np.abs(y - ref).max()))


@pytest.mark.parametrize("L_", [1, 7, 128, 129, 300, 2048])
@pytest.mark.parametrize("M", [3, 9])   # 3: split-key kernel; 9: one CTA per (row, head)
def test_attention_matches_fp64(pkg, L_, M):
    L = pkg.lib()
    H, T = 16, 2048
    rng = np.random.default_rng(L_)
    q = rng.standard_normal((M, H * 64)).astype(np.float32)
    k = (rng.standard_normal((M, H, T, 64)) * 0.5).astype(np.float16)
    v = rng.standard_normal((M, H, T, 64)).astype(np.float16)
    lens = np.array([[L_, max(1, L_ // 2), min(T, L_ + 5)][i % 3] for i in range(M)], np.int32)
    lens[M - 1] = max(1, min(T, lens[M - 1] - (M - 1)))
    kv = torch.from_numpy(np.stack([k, v])).cuda()   # [2][M][H][T][64]
    kd = kv[0]
    vd = kv[1]
    qd = torch.from_numpy(q).cuda()
    ld = torch.from_numpy(lens).cuda()
    od = torch.zeros((M, H * 64), dtype=torch.float32, device="cuda")
    # the op takes K and V bases of the same allocation (V = K + offset)
    pkg.check(L.t3b_op_attention(_p(qd), _p(kd), _p(vd), M, H, T, _p(ld), _p(od), _stream()))
    torch.cuda.synchronize()
    out = od.cpu().numpy()
    for m in range(M):
        for h in range(H):
            n = lens[m]
            s = (k[m, h, :n].astype(np.float64) @ q[m, h * 64:(h + 1) * 64].astype(np.float64)) / 8.0
            w = np.exp(s - s.max())
            ref = (w[:, None] * v[m, h, :n].astype(np.float64)).sum(0) / w.sum()
            assert rel_err(out[m, h * 64:(h + 1) * 64], ref) < 1e-5, (m, h, n)


@pytest.mark.parametrize("kind", ["narrow", "rounded"])
def test_sampler_bucket_and_radix_paths(pkg, orc, kind):
    """Top-k 1000 / top-p 0.95 without min-p on narrow logits (value bins
    hold few scores: the bucketed top-k + sort path) and on logits rounded to
    0.1 (thousands of exact ties: the radix-select + bitonic path): device
    tokens == oracle tokens."""
    L = pkg.lib()
    rows, V, HL = 128, 6563, 256
    rng = np.random.default_rng(11)
    if kind == "narrow":
        cond = np.stack([synth_logits(700 + r, scale=0.6) for r in range(rows)])
    else:
        cond = np.stack([synth_logits(700 + r, kind="rounded") for r in range(rows)])
    unc = np.zeros_like(cond)
    hist = rng.integers(0, V, (rows, HL)).astype(np.int32)
    hlen = np.full(rows, HL, np.int32)
    params = [dict(top_k=int(rng.choice([50, 1000])), top_p=float(rng.choice([0.8, 0.95, 1.0])), temp=0.8,
                   repeat_penalty=1.2, min_p=0.0, cfg_weight=0.0) for _ in range(rows)]
    seeds = rng.integers(0, 2 ** 63, rows, dtype=np.uint64)
    ctrs = rng.integers(0, 2 ** 40, rows, dtype=np.uint64)
    P = (pkg.SampleParams * rows)(*[pkg.SampleParams.make(**p) for p in params])
    pd = torch.frombuffer(bytearray(bytes(P)), dtype=torch.uint8).cuda()
    cd, ud = torch.from_numpy(cond).cuda(), torch.from_numpy(unc).cuda()
    hd, hld = torch.from_numpy(hist).cuda(), torch.from_numpy(hlen).cuda()
    sd = torch.from_numpy(seeds.view(np.int64)).cuda()
    ctd = torch.from_numpy(ctrs.view(np.int64)).cuda()
    td = torch.zeros(rows, dtype=torch.int32, device="cuda")
    pkg.check(L.t3b_op_sample_philox(_p(cd), _p(ud), rows, V, _p(hd), _p(hld), HL, _p(pd), _p(sd), _p(ctd),
                                     _p(td), _stream()))
    torch.cuda.synchronize()
    got = td.cpu().numpy()
    checked = 0
    for r in range(rows):
        x1, x2 = _philox_words(orc, int(seeds[r]), int(ctrs[r]), r)
        t, aux = orc.sample(cond[r], params[r], x1, x2, uncond=unc[r], hist=hist[r])
        if aux[2]:
            continue
        assert got[r] == t, (kind, r, params[r])
        checked += 1
    assert checked > rows // 2


def _philox_words(orc, seed, ctr, row):
    w = orc.philox([ctr & 0xFFFFFFFF, ctr >> 32, row, 0], [seed & 0xFFFFFFFF, seed >> 32])
    return int(w[0]), int(w[1])


def test_sampler_philox_matches_oracle(pkg, orc):
    """128 rows x 6563 (the sampler micro-benchmark shape) with CFG, min-p,
    penalty, top-k, top-p: device tokens == oracle tokens."""
    L = pkg.lib()
    rows, V, HL = 128, 6563, 256
    for trial in range(6):
        rng = np.random.default_rng(trial)
        cond = np.stack([synth_logits(10_000 * trial + r) for r in range(rows)])
        unc = np.stack([synth_logits(10_000 * trial + 5000 + r) for r in range(rows)])
        hist = rng.integers(0, V, (rows, HL)).astype(np.int32)
        hlen = rng.integers(0, HL + 1, rows).astype(np.int32)
        params = []
        for r in range(rows):
            params.append(dict(top_k=int(rng.choice([0, 50, 1000, 6563])), top_p=float(rng.choice([0.8, 0.95, 1.0])),
                               temp=float(rng.choice([0.0, 0.6, 0.8, 1.0])),
                               repeat_penalty=float(rng.choice([1.0, 1.2, 1.5])),
                               min_p=float(rng.choice([0.0, 0.05])), cfg_weight=float(rng.choice([0.0, 0.5]))))
        if trial == 0:   # the exact C2 configuration
            params = [dict(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2, min_p=0.05, cfg_weight=0.5)] * rows
            hlen[:] = HL
        seeds = rng.integers(0, 2 ** 63, rows, dtype=np.uint64)
        ctrs = rng.integers(0, 2 ** 40, rows, dtype=np.uint64)
        P = (pkg.SampleParams * rows)(*[pkg.SampleParams.make(**p) for p in params])
        pd = torch.frombuffer(bytearray(bytes(P)), dtype=torch.uint8).cuda()
        cd, ud = torch.from_numpy(cond).cuda(), torch.from_numpy(unc).cuda()
        hd, hld = torch.from_numpy(hist).cuda(), torch.from_numpy(hlen).cuda()
        sd = torch.from_numpy(seeds.view(np.int64)).cuda()
        ctd = torch.from_numpy(ctrs.view(np.int64)).cuda()
        td = torch.zeros(rows, dtype=torch.int32, device="cuda")
        pkg.check(L.t3b_op_sample_philox(_p(cd), _p(ud), rows, V, _p(hd), _p(hld), HL, _p(pd), _p(sd), _p(ctd),
                                         _p(td), _stream()))
        torch.cuda.synchronize()
        got = td.cpu().numpy()
        checked = 0
        for r in range(rows):
            x1, x2 = _philox_words(orc, int(seeds[r]), int(ctrs[r]), r)
            t, aux = orc.sample(cond[r], params[r], x1, x2, uncond=unc[r], hist=hist[r, :hlen[r]])
            if aux[2]:
                continue
            assert got[r] == t, (trial, r, params[r])
            checked += 1
        assert checked > rows * 0.9


@pytest.mark.parametrize("ties", [False, True])
def test_sampler_few_survivors_matches_oracle(pkg, orc, ties):
    """min-p leaves at most 32 scores: the one-warp path (top-k below the
    survivor count, top-p cuts, penalty, greedy and drawn rows; with `ties`
    the logits are rounded so equal scores meet the top-k threshold and the
    top-p order): device tokens == oracle tokens."""
    L = pkg.lib()
    rows, V, HL = 128, 6563, 64
    rng = np.random.default_rng(21 + ties)
    cond = np.stack([synth_logits(900 + r, scale=3.0, kind="rounded" if ties else "normal") for r in range(rows)])
    unc = np.zeros_like(cond)
    hist = rng.integers(0, V, (rows, HL)).astype(np.int32)
    hist[:, :8] = np.argsort(-cond, axis=1)[:, :8]          # the top scores are in the history
    hlen = rng.integers(0, HL + 1, rows).astype(np.int32)
    params = [dict(top_k=int(rng.choice([0, 1, 3, 8, 20, 1000])), top_p=float(rng.choice([0.3, 0.7, 0.95, 1.0])),
                   temp=float(rng.choice([0.0, 0.5, 0.8, 1.0])), repeat_penalty=float(rng.choice([1.0, 1.3])),
                   min_p=float(rng.choice([0.02, 0.05, 0.2])), cfg_weight=0.0) for _ in range(rows)]
    seeds = rng.integers(0, 2 ** 63, rows, dtype=np.uint64)
    ctrs = rng.integers(0, 2 ** 40, rows, dtype=np.uint64)
    P = (pkg.SampleParams * rows)(*[pkg.SampleParams.make(**p) for p in params])
    pd = torch.frombuffer(bytearray(bytes(P)), dtype=torch.uint8).cuda()
    cd, ud = torch.from_numpy(cond).cuda(), torch.from_numpy(unc).cuda()
    hd, hld = torch.from_numpy(hist).cuda(), torch.from_numpy(hlen).cuda()
    sd = torch.from_numpy(seeds.view(np.int64)).cuda()
    ctd = torch.from_numpy(ctrs.view(np.int64)).cuda()
    td = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ctr0 = ctd.clone()
    pkg.check(L.t3b_op_sample_philox(_p(cd), _p(ud), rows, V, _p(hd), _p(hld), HL, _p(pd), _p(sd), _p(ctd),
                                     _p(td), _stream()))
    torch.cuda.synchronize()
    got = td.cpu().numpy()
    drawn = (ctd - ctr0).cpu().numpy()
    few = checked = 0
    for r in range(rows):
        x1, x2 = _philox_words(orc, int(seeds[r]), int(ctrs[r]), r)
        t, aux = orc.sample(cond[r], params[r], x1, x2, uncond=unc[r], hist=hist[r, :hlen[r]])
        # a row draws once, unless it is greedy or nothing survived (then
        # the reference returns token 0 undrawn); the counter is the draw count
        assert drawn[r] in (0, 1) and (drawn[r] == 0 or params[r]["temp"] > 0.0), r
        if drawn[r] == 0 and params[r]["temp"] > 0.0:
            assert t == 0 and got[r] == 0, r
        if aux[2]:
            continue
        s = cond[r] / np.float32(params[r]["temp"]) if params[r]["temp"] not in (0.0, 1.0) else cond[r]
        few += int(np.count_nonzero(np.exp(s.astype(np.float64) - s.max()) >= params[r]["min_p"]) <= 32)
        assert got[r] == t, (r, params[r])
        checked += 1
    assert checked > rows * 0.8 and few > rows // 2, (checked, few)


def test_attention_length_error_is_reported(pkg):
    """A row whose length is 0 is skipped by the kernel and reported by
    t3b_op_check as T3B_ERR_DEVICE; the word is cleared by the read."""
    L = pkg.lib()
    M, H, T = 3, 16, 256
    q = torch.randn(M, H * 64, device="cuda")
    kv = torch.randn(2, M, H, T, 64, device="cuda").half()
    out = torch.zeros(M, H * 64, device="cuda")
    st = _stream()
    ok = torch.tensor([5, 7, 9], dtype=torch.int32, device="cuda")
    pkg.check(L.t3b_op_attention(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(ok), _p(out), st))
    assert L.t3b_op_check(st) == 0
    bad = torch.tensor([5, 0, 9], dtype=torch.int32, device="cuda")
    pkg.check(L.t3b_op_attention(_p(q), _p(kv[0]), _p(kv[1]), M, H, T, _p(bad), _p(out), st))
    assert L.t3b_op_check(st) == -5
    assert "length-out-of-range" in pkg.last_error()
    assert L.t3b_op_check(st) == 0


@pytest.mark.parametrize("M,p0", [(1, 0), (37, 0), (64, 0), (150, 0), (100, 900), (300, 1748)])
def test_prompt_attention_matches_fp64(pkg, M, p0):
    """Causal flash attention of a prompt chunk (t3b_op_attention_prompt):
    rows at positions p0 .. p0+M-1 of one cache, each over keys 0 .. its
    position, against the fp64 attention (1e-5 of max |out| per head)."""
    L = pkg.lib()
    H, T = 16, 2048
    rng = np.random.default_rng(M * 7 + p0)
    q = rng.standard_normal((M, H * 64)).astype(np.float32)
    k = (rng.standard_normal((H, T, 64)) * 0.5).astype(np.float16)
    v = rng.standard_normal((H, T, 64)).astype(np.float16)
    pos = (p0 + np.arange(M)).astype(np.int32)
    kv = torch.from_numpy(np.stack([k, v])).cuda()
    qd = torch.from_numpy(q).cuda()
    pd = torch.from_numpy(pos).cuda()
    od = torch.full((M, H * 64), float("nan"), dtype=torch.float32, device="cuda")
    pkg.check(L.t3b_op_attention_prompt(_p(qd), _p(kv[0]), _p(kv[1]), M, H, T, _p(pd), _p(od), _stream()))
    assert L.t3b_op_check(_stream()) == 0
    out = od.cpu().numpy()
    kf, vf = k.astype(np.float64), v.astype(np.float64)
    for m in range(0, M, max(1, M // 12)):
        n = int(pos[m]) + 1
        for h in range(H):
            s = (kf[h, :n] @ q[m, h * 64:(h + 1) * 64].astype(np.float64)) / 8.0
            w = np.exp(s - s.max())
            ref = (w[:, None] * vf[h, :n]).sum(0) / w.sum()
            assert rel_err(out[m, h * 64:(h + 1) * 64], ref) < 1e-5, (m, h, n)
