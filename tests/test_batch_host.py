"""Host side of the batched decode step, on the CPU: the tensor-core tile
layout of the weights and of the KV cache, the batch rules of the C ABI's
phase validation and the batch scratch size.  No kernel is launched."""
import numpy as np
import pytest
import torch

import _native
from batch_engine import kv_hf_layout, kv_store_tiles, kv_tiles, tile_weight


def test_tile_weight_layout():
    g = torch.Generator().manual_seed(0)
    n, k = 24, 4096
    w = torch.randn(n, k, generator=g).half()
    t = tile_weight(w)
    assert t.shape == (2, 3, 256, 8, 8)
    flat = t.reshape(-1)
    # element (row, col) sits in block (c, g) = (col // 2048, row // 8) at [column group][row][column]
    for row, col in [(0, 0), (7, 2047), (8, 2048), (23, 4095), (13, 3001), (16, 9)]:
        c, gg = col // 2048, row // 8
        v, e, r = (col % 2048) // 8, col % 8, row % 8
        off = ((c * (n // 8) + gg) * 256 + v) * 64 + r * 8 + e
        assert flat[off] == w[row, col], (row, col)
    # a block is its 8 x 2048 sub-matrix with rows interleaved per 8-column group
    blk = t[1, 2]  # rows 16..23, columns 2048..4095
    np.testing.assert_array_equal(blk.permute(1, 0, 2).reshape(8, 2048).numpy(), w[16:24, 2048:4096].numpy())
    # blocks are chunk-major (the K-blocked order of the batch-1 down_proj)
    assert torch.equal(t[0].reshape(-1), tile_weight(w[:, :2048].contiguous()).reshape(-1))


def test_tile_weight_rejects_bad_shapes():
    with pytest.raises(_native.AicasError):
        tile_weight(torch.zeros(12, 2048))
    with pytest.raises(_native.AicasError):
        tile_weight(torch.zeros(16, 1000))


def test_kv_tile_layout():
    """Slot p, dim d of a (layer, stream, head) slice sits at element
    (p // 8) * 1024 + (d // 8) * 64 + (p % 8) * 8 + d % 8 of the slice: the
    offsets the batched kernel's bulk copies, MMA descriptors and this
    step's k / v write use."""
    g = torch.Generator().manual_seed(3)
    L, B, H, M, D = 2, 3, 2, 64, 128
    cache = torch.zeros((L, B, H, M, D), dtype=torch.float16)
    P = 21  # a prompt that ends inside an 8-slot group
    P8 = 24
    src = torch.zeros((L, H, P8, D), dtype=torch.float16)
    src[:, :, :P] = torch.randn((L, H, P, D), generator=g).half()
    kv_store_tiles(cache, 1, src)
    flat = cache.view(L, B, H, M * D)
    for (l, h, p, d) in [(0, 0, 0, 0), (1, 1, 20, 127), (0, 1, 7, 8), (1, 0, 9, 63), (0, 0, 16, 65)]:
        off = (p // 8) * 1024 + (d // 8) * 64 + (p % 8) * 8 + d % 8
        assert flat[l, 1, h, off] == src[l, h, p, d], (l, h, p, d)
    hf = kv_hf_layout(cache)
    assert torch.equal(hf[:, 1, :, :P8], src)
    assert not hf[:, 1, :, P8:].any() and not hf[:, 0].any() and not hf[:, 2].any()
    # a 64-slot chunk is one contiguous 16 KB piece of its slice
    assert kv_tiles(cache)[0, 1, 0, :8].reshape(-1).data_ptr() == cache[0, 1, 0].data_ptr()


def test_batch_scratch_bytes():
    cta, b, heads, splits, hd = 256, 8, 8, 256, 128
    phases = 256
    header = 32 + 8 + 4 * phases  # shared words, launch counter, per-phase completion counters
    assert _native.batch_scratch_bytes() == header + cta * b * 4 * 2 + b * heads * splits * 2 * (hd + 1) * 8


def _gemv(**kw):
    p = _native.AicasPhase()
    p.kind, p.flags = _native.PH_GEMV, _native.F_LL_OUT
    p.n, p.k = 2048, 2048
    p.w = p.x = p.out = 4096
    for key, val in kw.items():
        setattr(p, key, val)
    return p


def _attn(**kw):
    p = _native.AicasPhase()
    p.kind, p.flags = _native.PH_ATTN, _native.F_LL_IN | _native.F_LL_OUT
    p.kv_heads, p.q_heads, p.max_len = 8, 16, 64
    p.k, p.n, p.x_src = 4096, 2048, 0
    p.x = p.out = p.k_cache = p.v_cache = p.norm_w = p.norm_w2 = 4096
    for key, val in kw.items():
        setattr(p, key, val)
    return p


def _check(*phases):
    return _native.lib().aicas_validate_batch_phases((_native.AicasPhase * len(phases))(*phases), len(phases))


def test_batch_validation_rules():
    ll_in = _native.F_LL_OUT | _native.F_LL_IN
    assert _check(_gemv()) == 0
    assert _check(_gemv(n=2044)) == 2  # rows: whole 8-row tiles
    assert _check(_gemv(k=1024)) == 2  # columns: whole 2048-column tiles
    assert _check(_gemv(k=6144)) == 2  # k > 2048 must be K-blocked
    assert _check(_gemv(k=6144, flags=_native.F_LL_OUT | _native.F_KBLOCKED)) == 0
    assert _check(_gemv(flags=0)) == 1  # outputs are LL vectors
    assert _check(_gemv(w=4100)) == 3
    assert _check(_gemv(flags=_native.F_LL_OUT | _native.F_BARRIER)) == 1
    assert _check(_gemv(flags=ll_in, x_src=0)) == 1  # an LL input comes from an earlier phase
    assert _check(_gemv(), _gemv(flags=ll_in, x_src=0)) == 0
    assert _check(_gemv(kind=_native.PH_GATEUP, k=4096, flags=_native.F_LL_OUT | _native.F_KBLOCKED)) == 1
    assert _check(_gemv(), _attn()) == 0
    assert _check(_gemv(), _attn(k=2048)) == 2  # x row length = q + k + v of a stream
    assert _check(_gemv(), _attn(flags=_native.F_LL_IN | _native.F_LL_OUT | _native.F_Q_READY)) == 1
    assert _check(_gemv(), _attn(q_heads=8)) == 2
    # counted vectors: an input must come from a phase that writes one
    cnt = _native.F_CNT_OUT
    assert _check(_gemv(flags=cnt), _gemv(flags=cnt | _native.F_CNT_IN, x_src=0)) == 0
    assert _check(_gemv(), _gemv(flags=cnt | _native.F_CNT_IN, x_src=0)) == 1  # source writes LL words
    assert _check(_gemv(flags=cnt), _gemv(flags=_native.F_LL_OUT | _native.F_LL_IN, x_src=0)) == 1
    assert _check(_gemv(flags=cnt | _native.F_LL_OUT)) == 1  # one output kind
    assert _check(_gemv(), _attn(flags=_native.F_LL_IN | cnt)) == 0


def _operand(buf: np.ndarray, base: int, rows: int, lbo: int, sbo: int) -> np.ndarray:
    """The [rows x 16] fp16 matrix a K-major no-swizzle shared-memory
    descriptor (start `base` bytes into `buf`, K-adjacent core matrices `lbo`
    bytes apart, 8-row groups `sbo` bytes apart) hands the tensor core for one
    K = 16 step: element (m, k) at base + (m / 8) sbo + (k / 8) lbo + (m % 8) 16 + (k % 8) 2."""
    m = np.arange(rows)[:, None]
    k = np.arange(16)[None, :]
    addr = base + (m // 8) * sbo + (k // 8) * lbo + (m % 8) * 16 + (k % 8) * 2
    return buf[addr // 2]


def test_block_pair_mma_reproduces_the_projection():
    """Emulates, in numpy, how decode_batch.cu's tensor cores read one weight
    tile and the streams' operand: 8 K steps of M = 128, N = 128, K = 16 with
    the tile and the operand described as canonical K-major layouts (LBO =
    128 B, SBO = 2 KB, 256 bytes per K step), accumulating D[(j, r)][(j', s)];
    the sum of D's 16 diagonal blocks j == j' must be the tile's 8 rows times
    the 8 streams (W x^T)."""
    g = torch.Generator().manual_seed(7)
    w = torch.randn(8, 2048, generator=g).half()
    x = torch.randn(8, 2048, generator=g).half()  # 8 streams
    tile = tile_weight(w).reshape(-1).numpy()      # one 32 KB tile, the kernel's ring stage
    xa = tile_weight(x).reshape(-1).numpy()        # the streams' operand uses the same layout
    d = np.zeros((128, 128), dtype=np.float64)
    for ks in range(8):
        a = _operand(tile, 256 * ks, 128, 128, 2048).astype(np.float64)
        b = _operand(xa, 256 * ks, 128, 128, 2048).astype(np.float64)
        d += a @ b.T
    out = sum(d[8 * j:8 * j + 8, 8 * j:8 * j + 8] for j in range(16))  # rows r, columns s
    ref = w.double().numpy() @ x.double().numpy().T
    np.testing.assert_allclose(out, ref, rtol=1e-9, atol=1e-9)
    # the off-diagonal blocks are the products the epilogue discards
    assert np.abs(d[0:8, 8:16]).max() > 0


def _operand_mn(buf: np.ndarray, base: int, cols: int, lbo: int, sbo: int) -> np.ndarray:
    """The [16 x cols] fp16 matrix (K = 16 rows, MN = cols) an MN-major
    no-swizzle descriptor hands the tensor core for one K step: core matrices
    of 8 K-rows x 8 MN-elements (16 bytes per K-row), 8-deep K groups `lbo`
    bytes apart, 8-wide MN blocks `sbo` bytes apart: element (k, n) at
    base + (k / 8) lbo + (n / 8) sbo + (k % 8) 16 + (n % 8) 2."""
    k = np.arange(16)[:, None]
    n = np.arange(cols)[None, :]
    addr = base + (k // 8) * lbo + (n // 8) * sbo + (k % 8) * 16 + (n % 8) * 2
    return buf[addr // 2]


def test_attention_mma_operands_over_the_kv_tile_layout():
    """Emulates the tensor-core attention of decode_batch.cu (and, with 128-row
    blocks, of prefill_attn_tc.cu) on a K / V tile stored in the KV tile
    layout: S = K Q^T with both operands K-major (LBO 128 B, SBO 2 KB, 256 bytes
    per 16-dim K step) and O = V^T P^T with V read MN-major (LBO 2 KB along the
    slots, SBO 128 B along the dims, 4096 bytes per 16-slot K step) and P
    K-major (LBO 128 B, SBO 1 KB for 64 slots).  The same conventions were
    checked exact on a B200 by a probe."""
    g = torch.Generator().manual_seed(11)
    L, D = 64, 128
    k = torch.randn(L, D, generator=g).half()
    v = torch.randn(L, D, generator=g).half()
    q = torch.randn(2, D, generator=g).half()       # the KV head's two query heads
    p = torch.rand(2, L, generator=g).half()        # probabilities
    cache = torch.zeros((1, 1, 1, L, D), dtype=torch.float16)
    kv_store_tiles(cache, 0, k.view(1, 1, L, D))
    ktile = cache.reshape(-1).numpy().copy()
    kv_store_tiles(cache, 0, v.view(1, 1, L, D))
    vtile = cache.reshape(-1).numpy().copy()
    # queries: B operand [16 rows x 128 dims], rows 2.. zero; layout (n/8) 2048 + (d/8) 128 + (n%8) 16 + (d%8) 2
    qop = np.zeros(16 * D, dtype=np.float16)
    for n in range(2):
        for d in range(D):
            qop[((n // 8) * 2048 + (d // 8) * 128 + (n % 8) * 16 + (d % 8) * 2) // 2] = q[n, d].item()
    s = np.zeros((L, 16))
    for ks in range(D // 16):
        a = _operand(ktile, 256 * ks, L, 128, 2048).astype(np.float64)
        b = _operand(qop, 256 * ks, 16, 128, 2048).astype(np.float64)
        s += a @ b.T
    np.testing.assert_allclose(s[:, :2], k.double().numpy() @ q.double().numpy().T, rtol=1e-9, atol=1e-9)
    assert not s[:, 2:].any()
    # probabilities: B operand [16 rows x 64 slots], K-major, row g at (g/8) 1024 + (r/8) 128 + (g%8) 16 + (r%8) 2
    pop = np.zeros(16 * L, dtype=np.float16)
    for n in range(2):
        for r in range(L):
            pop[((n // 8) * 1024 + (r // 8) * 128 + (n % 8) * 16 + (r % 8) * 2) // 2] = p[n, r].item()
    o = np.zeros((D, 16))
    for ks in range(L // 16):
        a = _operand_mn(vtile, 4096 * ks, D, 2048, 128).astype(np.float64).T  # A = V^T: [128 dims x 16 slots]
        b = _operand(pop, 256 * ks, 16, 128, 1024).astype(np.float64)          # B = P: [16 rows x 16 slots]
        o += a @ b.T
    np.testing.assert_allclose(o[:, :2], v.double().numpy().T @ p.double().numpy().T, rtol=1e-9, atol=1e-9)
