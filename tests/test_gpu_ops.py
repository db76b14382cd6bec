"""GPU parity of every operator entry point against the CPU oracle.

Tolerances: integer/byte work (dequant, quantiser, KV write, residual add,
sampled ids) is bit-exact.  fp16 outputs of reductions may differ from the
oracle by the rounding of a differently ordered fp32 sum: |d| <= 2 ulp(fp16)
of the value plus 1e-4 absolute, and >= 95% of elements bit-exact.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qweninferenceengine_b200 import ops  # noqa: E402


def T(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def N(t):
    return t.cpu().numpy()


def ulp16(x):
    x = np.abs(x.astype(np.float32))
    e = np.floor(np.log2(np.maximum(x, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def assert_close16(gpu, ref, ulps=2, abs_tol=1e-4, min_exact=0.95):
    g = np.asarray(gpu, np.float16).astype(np.float32)
    r = np.asarray(ref, np.float16).astype(np.float32)
    d = np.abs(g - r)
    lim = ulps * ulp16(r) + abs_tol
    bad = np.nonzero(d > lim)[0]
    assert bad.size == 0, f"{bad.size} elements off; worst {d.max()} at {d.argmax()} ({g[d.argmax()]} vs {r[d.argmax()]})"
    exact = np.mean(np.asarray(gpu, np.float16).view(np.uint16) == np.asarray(ref, np.float16).view(np.uint16))
    assert exact >= min_exact, f"only {exact:.3f} bit-exact"


def q4_config1(seed, n, k):
    """Config 1: q uniform in [-8,7] stored as q+8, scales |N(0,0.02)|/7 per block."""
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(n, k), dtype=np.uint8)
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    scales = (np.abs(rng.standard_normal(n * k // 32)) * 0.02 / 7).astype(np.float16)
    x = rng.standard_normal(k).astype(np.float16)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float16)
    return packed, scales, x, bias


def test_dequant_all_bytes_bitexact(cuda, oracle):
    # every byte value in every nibble position, with a spread of scales
    b = np.arange(256, dtype=np.uint8)
    packed = np.tile(b, 64)                     # 16384 bytes = 32768 weights
    rng = np.random.default_rng(1)
    scales = (np.abs(rng.standard_normal(packed.size * 2 // 32)) * 0.05).astype(np.float16)
    scales[:4] = [1.0, 0.0, 65504.0, 6e-8]
    ref = oracle.dequant_q4(packed, scales, packed.size * 2)
    got = N(ops.dequant_q4(T(packed), T(scales), packed.size * 2))
    assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("n,k,seed", [(8960, 1536, 0), (1536, 8960, 1), (37, 1536, 2), (5, 64, 3)])
def test_gemv_q4_0(cuda, oracle, n, k, seed):
    packed, scales, x, bias = q4_config1(seed, n, k)
    ref = oracle.gemv_q4_0(packed, scales, x, bias)
    got = N(ops.gemv_q4_0(T(packed), T(scales), T(x), T(bias)))
    assert_close16(got, ref)
    ref0 = oracle.gemv_q4_0(packed, scales, x, None)
    got0 = N(ops.gemv_q4_0(T(packed), T(scales), T(x), None))
    assert_close16(got0, ref0)


def test_gemv_fp16(cuda, oracle):
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((4099, 1536)) * 0.02).astype(np.float16)
    x = rng.standard_normal(1536).astype(np.float16)
    assert_close16(N(ops.gemv_fp16(T(w), T(x))), oracle.gemv_fp16(w, x))


def test_rms_norm(cuda, oracle):
    rng = np.random.default_rng(5)
    for scale in (0.01, 1.0, 40.0):
        x = (rng.standard_normal(1536) * scale).astype(np.float16)
        g = (1 + rng.standard_normal(1536) * 0.02).astype(np.float16)
        assert_close16(N(ops.rms_norm_q4(T(x), T(g))), oracle.rms_norm(x, g), min_exact=0.97)


@pytest.mark.parametrize("sl", [1, 2, 512, 1024, 8704])
def test_rope(cuda, oracle, sl):
    rng = np.random.default_rng(sl)
    q = rng.standard_normal(1536).astype(np.float16)
    slt = T(np.array([sl], np.uint32).view(np.int32))
    got = N(ops.apply_rope_q4(T(q), 12, slt))
    assert_close16(got, oracle.rope(q, 12, sl), ulps=1, min_exact=0.97)


def test_write_kv_and_elementwise(cuda, oracle):
    rng = np.random.default_rng(6)
    kk = rng.standard_normal(256).astype(np.float16)
    vv = rng.standard_normal(256).astype(np.float16)
    kc = np.zeros((64, 256), np.float16)
    vc = np.zeros((64, 256), np.float16)
    kct, vct = T(kc), T(vc)
    ops.write_kv_cache(T(kk), T(vv), kct, vct, T(np.array([9], np.int32)), 64)
    oracle.write_kv_cache(kk, vv, kc, vc, 9)
    assert np.array_equal(N(kct).view(np.uint16), kc.view(np.uint16))
    assert np.array_equal(N(vct).view(np.uint16), vc.view(np.uint16))
    # guard: positions >= max_ctx are skipped
    ops.write_kv_cache(T(kk), T(vv), kct, vct, T(np.array([65], np.int32)), 64)
    assert np.array_equal(N(kct).view(np.uint16), kc.view(np.uint16))
    a = (rng.standard_normal(1536) * 5).astype(np.float16)
    b = (rng.standard_normal(1536) * 5).astype(np.float16)
    assert np.array_equal(N(ops.residual_add(T(a), T(b))).view(np.uint16),
                          oracle.residual_add(a, b).view(np.uint16))
    gate = np.concatenate([rng.standard_normal(8950) * 8, [15, 15.01, -15, -15.01, 16, -16, 0, 30, -30, 1e-3]]).astype(np.float16)
    up = rng.standard_normal(8960).astype(np.float16)
    got = N(ops.swiglu(T(gate), T(up)))
    assert_close16(got, oracle.swiglu(gate, up), ulps=1, abs_tol=0, min_exact=0.99)


def test_quantizer_bitexact(cuda, oracle):
    rng = np.random.default_rng(8)
    w = rng.standard_normal(1536 * 96, dtype=np.float32) * 0.02
    w[:32] = 0.0                        # scale 0 block
    w[32:64] = np.linspace(-1, 1, 32)   # exact halves -> round half away from zero
    p_ref, s_ref = oracle.quantize_q4(w)
    p, s = ops.quantize_q4(T(w))
    assert np.array_equal(N(p), p_ref)
    assert np.array_equal(N(s).view(np.uint16), s_ref.view(np.uint16))


@pytest.mark.parametrize("L", [1, 17, 512, 1024, 8704])
def test_attention(cuda, oracle, L):
    rng = np.random.default_rng(L)
    max_ctx = max(L, 64) + 3
    q = rng.standard_normal(1536).astype(np.float16)
    kc = rng.standard_normal((max_ctx, 256)).astype(np.float16)
    vc = rng.standard_normal((max_ctx, 256)).astype(np.float16)
    ref = oracle.attention(q, kc, vc, L)
    sl = T(np.array([L], np.int32))
    qt, kt, vt = T(q), T(kc), T(vc)
    fused = N(ops.attention_decode(qt, kt, vt, sl, max_ctx))
    assert_close16(fused, ref, min_exact=0.9)
    scores = torch.zeros(12 * max_ctx, dtype=torch.float32, device="cuda")
    out = torch.zeros(1536, dtype=torch.float16, device="cuda")
    ops.attention_scores(qt, kt, scores, sl, max_ctx)
    ops.softmax(scores, sl)
    ops.attn_weighted_sum(scores, vt, out, sl)
    assert_close16(N(out), ref, min_exact=0.9)


def test_sampler_greedy(cuda, oracle):
    rng = np.random.default_rng(9)
    lg = (rng.standard_normal((4, 151936)) * 2).astype(np.float16)
    lg[1, 5000] = lg[1, 7000] = 40.0           # tie -> first index
    lg[2, :] = np.nan                          # all NaN -> 151645
    lg[3, ::2] = np.nan
    got = N(ops.sample(T(lg), 0.0, 0.9))
    want = [oracle.sample_greedy(lg[i]) for i in range(4)]
    assert got.tolist() == want
    assert want[1] == 5000 and want[2] == 151645


@pytest.mark.parametrize("temp,top_p", [(0.7, 0.9), (0.7, 0.8), (1.0, 1.0), (0.3, 0.0), (2.0, 0.5)])
def test_sampler_top_p_bitexact(cuda, oracle, temp, top_p):
    rng = np.random.default_rng(int(temp * 100 + top_p * 10))
    n = 12
    lg = (rng.standard_normal((n, 151936)) * rng.uniform(0.05, 6, size=(n, 1))).astype(np.float16)
    lg[0, :100] = 3.0                  # ties in the nucleus
    lg[1, 10] = np.nan                 # NaN quirk
    lg[2, :] = lg[2, 0]                # all equal
    u = np.array([oracle.uniform24(3, i, 17) for i in range(n)], np.uint32)
    u[3] = 0
    u[4] = (1 << 24) - 1
    got = N(ops.sample(T(lg), temp, top_p, T(u.view(np.int32))))
    want = [oracle.sample_top_p(lg[i], temp, top_p, int(u[i])) for i in range(n)]
    assert got.tolist() == want


@pytest.mark.parametrize("vocab", [151936, 151666, 4099, 1])
def test_sampler_grid_bitexact(cuda, oracle, vocab):
    """One sequence over every SM (qwen_sample_scratch, the batch-1 engine
    step's sampler; digit totals exchanged through device memory): the
    oracle's ids on flat, peaked, tied, all-equal, NaN and all-NaN rows, with
    u24 and top_p at their ends, and the scratch back at zero after every
    call.  The all-equal row puts the draw in a tie group spread over every
    CTA (the per-CTA counts go through one more barrier); 4,099 ids leave the
    last CTAs none."""
    rng = np.random.default_rng(vocab)
    rows = [(rng.standard_normal(151936) * sc).astype(np.float16) for sc in (0.05, 0.5, 1.0, 3.0, 8.0)]
    r = rng.standard_normal(151936).astype(np.float16)
    r[:100] = 3.0                       # ties in the nucleus
    rows.append(r)
    r = rng.standard_normal(151936).astype(np.float16)
    r[10] = np.nan                      # NaN quirk
    rows.append(r)
    rows.append(np.full(151936, 0.25, np.float16))
    rows.append(np.full(151936, np.nan, np.float16))
    scr = ops.sample_scratch(1, "cuda")
    assert scr is not None and ops.sample_scratch(4, "cuda") is None
    for i, lg in enumerate(rows):
        for temp, top_p, u in ((0.7, 0.8, oracle.uniform24(5, i, 9)), (1.0, 1.0, 0),
                               (0.3, 0.0, (1 << 24) - 1), (0.7, 0.95, (1 << 24) - 1)):
            uu = T(np.array([u], np.uint32).view(np.int32))
            got = int(N(ops.sample(T(lg[None, :]), temp, top_p, uu, vocab=vocab, scratch=scr))[0])
            want = oracle.sample_top_p(lg, temp, top_p, int(u), vocab=vocab)
            assert got == want, (i, temp, top_p, u)
            assert not N(scr).any(), (i, temp, top_p, u)
    # greedy with a scratch runs the cluster path
    if vocab <= 151666:
        got = N(ops.sample(T(rows[3][None, :]), 0.0, 0.9, vocab=vocab, scratch=scr))
        assert got.tolist() == [oracle.sample_greedy(rows[3][:vocab])]


@pytest.mark.parametrize("n", [1, 3, 12, 17, 64])
def test_sampler_batch_sizes_bitexact(cuda, oracle, n):
    """Batches run on 16-, 8- or 4-CTA clusters by size (the largest cluster
    whose one wave holds the batch, else 4): every size draws the oracle's ids
    (flat and peaked rows, u24 at both ends), greedy included."""
    rng = np.random.default_rng(100 + n)
    lg = (rng.standard_normal((n, 151936)) * rng.uniform(0.1, 5, size=(n, 1))).astype(np.float16)
    u = np.array([oracle.uniform24(11, i, 5) for i in range(n)], np.uint32)
    u[0] = (1 << 24) - 1
    if n > 1:
        u[1] = 0
    for temp, top_p in ((0.7, 0.8), (1.0, 0.95)):
        got = N(ops.sample(T(lg), temp, top_p, T(u.view(np.int32))))
        want = [oracle.sample_top_p(lg[i], temp, top_p, int(u[i])) for i in range(n)]
        assert got.tolist() == want
    lg[0, 7] = lg[0].max() + 1.0
    got = N(ops.sample(T(lg), 0.0, 0.9))
    assert got.tolist() == [oracle.sample_greedy(lg[i]) for i in range(n)]
