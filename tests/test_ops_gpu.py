"""GPU parity of the single-op entry points against the CPU oracle.

Each test calls the drop-in Python names (which call the C ABI) and compares
with the oracle on the same seeded inputs.  Tolerances: fp16 outputs must
agree to within 2 fp16 ulps of the value (|d| <= 2^-9 * max(1, |ref|)),
i.e. the only difference allowed is fp32 accumulation order.
"""
import numpy as np
import pytest
import torch

from oracle.qwen3vl_oracle import (attention_reference, gemv_reference, post_attn_mlp_reference, rms_norm,
                                   rope)

pytestmark = pytest.mark.gpu

ULP2 = 2.0 ** -9


def _close16(got, ref):
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    tol = ULP2 * np.maximum(1.0, np.abs(ref)) + 1e-6
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} mismatches, max |d| {np.abs(got - ref).max()}"


def _randn(shape, seed, scale=1.0, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).half().to(dev)


@pytest.mark.parametrize("n,k", [(4096, 2048), (2048, 2048), (12288, 2048), (2048, 6144), (1000, 8),
                                 (5, 4104), (151936, 2048), (301, 4096), (77, 2056), (3, 6144)])
def test_gemv_matches_oracle(cuda_device, n, k):
    import cuda_decode_gemv as cg

    w = _randn((n, k), 1, 0.02)
    x = _randn((1, 1, k), 2)
    y = cg.nosplit_matvec_half(x, w, None)
    assert y.shape == (1, 1, n)
    ref = gemv_reference(w.float().cpu().numpy(), x.reshape(-1).float().cpu().numpy())
    _close16(y.reshape(-1).float().cpu().numpy(), ref)


def test_gemv_bias_and_repeat_calls(cuda_device):
    import cuda_decode_gemv as cg

    w = _randn((3000, 2048), 3, 0.02)
    x = _randn((1, 1, 2048), 4)
    b = _randn((3000,), 5, 0.1)
    ws = {"type": "nosplit", "out": torch.empty(3000, dtype=torch.float16, device="cuda")}
    for _ in range(3):  # scratch reuse across launches
        y = cg.nosplit_matvec_half(x, w, b, workspace=ws)
    assert y.data_ptr() == ws["out"].data_ptr()
    ref = w.float().cpu().numpy() @ x.reshape(-1).float().cpu().numpy() + b.float().cpu().numpy()
    _close16(y.reshape(-1).float().cpu().numpy(), ref.astype(np.float16).astype(np.float32))


def test_fused_rmsnorm_qkv(cuda_device):
    import cuda_decode_gemv as cg

    x = _randn((1, 1, 2048), 6, 3.0)
    nw = (1 + _randn((2048,), 7, 0.1))
    w = _randn((4096, 2048), 8, 0.02)
    y = cg.fused_rmsnorm_qkv_half(x, nw, w, None, 1e-6)
    xn = rms_norm(x.reshape(-1).float().cpu().numpy(), nw.float().cpu().numpy(), 1e-6)
    ref = gemv_reference(w.float().cpu().numpy(), xn)
    _close16(y.reshape(-1).float().cpu().numpy(), ref)


def test_post_attn_mlp(cuda_device):
    import cuda_decode_gemv as cg

    r = _randn((1, 1, 2048), 9, 2.0)
    a = _randn((1, 1, 2048), 10, 1.0)
    nw = 1 + _randn((2048,), 11, 0.1)
    wgu = _randn((12288, 2048), 12, 0.02)
    wd = _randn((2048, 6144), 13, 0.02)
    act, out = cg.fused_post_attn_mlp_softsync_half(r, a, nw, wgu, wd, None, 1e-6)
    assert act.shape == (1, 1, 6144) and out.shape == (1, 1, 2048)
    f = lambda t: t.reshape(-1).float().cpu().numpy()
    ract, rout = post_attn_mlp_reference(f(r), f(a), f(nw), wgu.float().cpu().numpy(), wd.float().cpu().numpy())
    _close16(f(act), ract)
    # `out` depends on act through a 6144-long dot: allow act's own rounding flips
    assert np.abs(f(out) - rout).max() <= 4e-3 * max(1.0, np.abs(rout).max())


@pytest.mark.parametrize("L", [1, 31, 32, 33, 128, 777, 1024, 4096, 8192])
def test_decode_attention_splitkv(cuda_device, L):
    import cuda_decode_attention as ca

    lmax = 8192
    q = _randn((1, 16, 1, 128), 20 + L)
    k = _randn((1, 8, lmax, 128), 21 + L)
    v = _randn((1, 8, lmax, 128), 22 + L)
    pos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
    out = ca.decode_attn_v4_cta_qhead_splitkv_fused(q, k, v, 128 ** -0.5, 2, pos)
    assert out.shape == (1, 1, 16, 128)
    ref = attention_reference(q.reshape(16, 128).float().cpu().numpy(), k[0, :, :L].float().cpu().numpy(),
                              v[0, :, :L].float().cpu().numpy(), L, 128 ** -0.5)
    got = out.reshape(16, 128).float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-3


@pytest.mark.parametrize("kvh,lmax,L", [(1, 1000, 1000), (4, 1000, 129), (2, 4100, 4100), (8, 300, 2)])
def test_decode_attention_other_head_counts_and_cache_sizes(cuda_device, kvh, lmax, L):
    """The split-KV op with 1, 2, 4 or 8 KV heads (two query heads each) and
    caches whose length is no multiple of the 128-slot chunk, through the C ABI:
    against attention_reference, and a second call equal to the first (the
    merge counters return to zero)."""
    import ctypes

    import _native

    lib = _native.lib()
    q = _randn((2 * kvh, 128), 40 + kvh)
    k = _randn((kvh, lmax, 128), 41 + kvh)
    v = _randn((kvh, lmax, 128), 42 + kvh)
    pos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
    scratch = torch.zeros(_native.scratch_bytes(), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        out = torch.full((2 * kvh, 128), float("nan"), dtype=torch.float16, device="cuda")
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _native.check(lib.aicas_decode_attn_splitkv_f16(p(q), p(k), p(v), p(pos), 128 ** -0.5, p(out), 2 * kvh, kvh,
                                                        lmax, p(scratch),
                                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                      "aicas_decode_attn_splitkv_f16")
        outs.append(out)
    ref = attention_reference(q.float().cpu().numpy(), k[:, :L].float().cpu().numpy(), v[:, :L].float().cpu().numpy(),
                              L, 128 ** -0.5)
    assert np.abs(outs[0].float().cpu().numpy() - ref).max() <= 2e-3
    assert torch.equal(outs[0], outs[1])


def test_decode_attention_rejects_bad_gqa(cuda_device):
    import cuda_decode_attention as ca

    q = _randn((1, 16, 1, 128), 1)
    k = _randn((1, 4, 64, 128), 2)
    pos = torch.tensor([3], dtype=torch.int64, device="cuda")
    assert ca.decode_attn_v4_cta_qhead_splitkv_fused(q, k, k, 0.1, 4, pos) is None


def test_q_rope_kv_cache_update(cuda_device):
    import cuda_decode_small_ops as cs

    q = _randn((1, 1, 16, 128), 30, 2.0)
    k = _randn((1, 1, 8, 128), 31, 2.0)
    v = _randn((1, 1, 8, 128), 32)
    qw = 1 + _randn((128,), 33, 0.1)
    kw = 1 + _randn((128,), 34, 0.1)
    ang = torch.arange(128, dtype=torch.float32) * 0.37
    cos = torch.cos(ang).half().view(1, 1, 128).cuda()
    sin = torch.sin(ang).half().view(1, 1, 128).cuda()
    kc = torch.zeros((1, 8, 64, 128), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    pos = torch.tensor([17], dtype=torch.int64, device="cuda")
    qo = cs.fused_q_rope_kv_cache_update(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, pos)
    f = lambda t: t.float().cpu().numpy()
    c, s_ = f(cos).reshape(1, 128), f(sin).reshape(1, 128)
    rq = rope(rms_norm(f(q).reshape(1, 16, 128), f(qw), 1e-6), c, s_)
    rk = rope(rms_norm(f(k).reshape(1, 8, 128), f(kw), 1e-6), c, s_)
    _close16(f(qo).reshape(1, 16, 128), rq)
    _close16(f(kc[0, :, 17]), rk[0])
    np.testing.assert_array_equal(f(vc[0, :, 17]), f(v).reshape(8, 128))
    assert float(kc[0, :, :17].abs().sum()) == 0 and float(kc[0, :, 18:].abs().sum()) == 0


def test_lm_head_argmax(cuda_device):
    import cuda_decode_gemv as cg

    w = _randn((151936, 2048), 40, 0.02)
    x = _randn((1, 1, 2048), 41)
    logits, tok = cg.lm_head_argmax_half(x, w)
    lg = logits.reshape(-1).float().cpu().numpy()
    assert int(tok.reshape(-1)[0]) == int(np.argmax(lg))  # first max of the fp16 logits
    ref = gemv_reference(w.float().cpu().numpy(), x.reshape(-1).float().cpu().numpy())
    _close16(lg, ref)
    # planted tie: two rows identical to the max row -> the smallest index wins
    best = int(np.argmax(lg))
    w[7] = w[best]
    w[151935] = w[best]
    _, tok2 = cg.lm_head_argmax_half(x, w, return_logits=False)
    assert int(tok2.reshape(-1)[0]) == min(7, best)
