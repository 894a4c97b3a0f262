"""CUDA kernels vs the oracle, through the C ABI (libdiolkos.so).

Bit-exact: both quantisers, the int32 group dots, packing, and the GEMV output itself (the
kernel replays the reference's group order and rounding).  Tolerance: rmsnorm (2 ulp-level; the
reduction order differs)."""
import hashlib
import os

import numpy as np
import pytest

from diolkos_b200 import synth
from tests.golden import make_golden as G

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    torch.cuda.init()
    return torch


@pytest.fixture(scope="module")
def kgold():
    return np.load(os.path.join(GOLD, "kernels.npz"))


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("case", G.QUANT_F32_CASES)
def test_quant_f32_bit_exact(torch_cuda, port, kgold, case):
    from diolkos_b200 import ops

    seed, n, sc = case
    x = G.quant_f32_input(seed, n, sc)
    q, s = ops.quantize_f32(_dev(torch_cuda, x))
    q, s = q.cpu().numpy(), s.cpu().numpy()
    assert sha(q) == str(kgold[f"qf32_{seed}_q"]) and sha(s) == str(kgold[f"qf32_{seed}_s"])
    pq, ps = port.quant_f32(x)
    np.testing.assert_array_equal(q, pq)


@pytest.mark.parametrize("case", G.QUANT_BF16_CASES)
def test_quant_bf16_bit_exact(torch_cuda, port, kgold, case):
    from diolkos_b200 import ops

    seed, n, sc = case
    x = G.quant_bf16_input(seed, n, sc)
    q, s = ops.quantize_bf16(_dev(torch_cuda, x.view(np.int16)))
    q, s = q.cpu().numpy(), s.cpu().numpy()
    assert sha(q) == str(kgold[f"qbf16_{seed}_q"]) and sha(s) == str(kgold[f"qbf16_{seed}_s"])


def test_quant_edge_groups(torch_cuda, port):
    """Zero groups, one-hot groups, denormals, huge values, exact ties -- GPU == oracle."""
    from diolkos_b200 import ops

    rng = np.random.default_rng(1)
    groups = [np.zeros(32, np.float32), np.eye(1, 32, 5, dtype=np.float32)[0] * -3.0,
              np.full(32, 1e-40, np.float32), rng.standard_normal(32).astype(np.float32) * 1e30,
              np.linspace(-127, 127, 32, dtype=np.float32), np.array([2.5, 3.5, -2.5, 127.0] * 8, np.float32)]
    x = np.concatenate(groups)
    q, s = ops.quantize_f32(_dev(torch_cuda, x))
    pq, ps = port.quant_f32(x)
    np.testing.assert_array_equal(q.cpu().numpy(), pq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), ps.view(np.uint32))


def test_group_dots_exact(torch_cuda, port):
    from diolkos_b200 import ops

    rng = np.random.default_rng(2)
    for n, d in [(4096, 64), (11008, 8), (288, 33)]:
        xq = rng.integers(-127, 128, n, dtype=np.int8)
        wq = rng.integers(-128, 128, n * d, dtype=np.int8)
        dots = ops.group_dots(_dev(torch_cuda, xq), _dev(torch_cuda, wq), n, d).cpu().numpy()
        np.testing.assert_array_equal(dots, port.group_dots(xq, wq, n, d))


def _row_bytes(n):
    """Bytes of one packed row: per 512-column block, values + scales padded to 16 bytes."""
    blk = lambda w: (w + w // 8 + 15) // 16 * 16
    return (n // 512) * 576 + (blk(n % 512) if n % 512 else 0)


def _unpack(w, n, d, T):
    """Decode the tile layout (restated from diolkos_b200/csrc/dk_kernels.h): tile t of T rows stores
    block b of its rows at t*T*row_bytes + T*576*b, row r of the tile at + r*blk_bytes(w_b); inside a
    segment value chunk c sits at c ^ (r & 7) (when w_b/16 is a multiple of 8) and scale chunk s at
    s ^ ((r >> 1) & 3) (w_b == 512) or s ^ (r & 1) (w_b == 256)."""
    rb = _row_bytes(n)
    q = np.empty((d, n), np.int8)
    sc = np.empty((d, n // 32), np.float32)
    for row in range(d):
        t, r = divmod(row, T)
        for b in range((n + 511) // 512):
            wb = min(512, n - 512 * b)
            bb = (wb + wb // 8 + 15) // 16 * 16
            off = t * T * rb + T * 576 * b + r * bb
            seg = w[off:off + bb]
            for c in range(wb // 16):
                pc = c ^ (r & 7) if (wb // 16) % 8 == 0 else c
                q[row, 512 * b + 16 * c:512 * b + 16 * c + 16] = seg[16 * pc:16 * pc + 16].view(np.int8)
            for g in range(wb // 32):
                s4 = g >> 2
                ps = s4 ^ ((r >> 1) & 3) if wb == 512 else (s4 ^ (r & 1) if wb == 256 else s4)
                o = wb + 16 * ps + 4 * (g & 3)
                sc[row, 16 * b + g] = seg[o:o + 4].view(np.float32)[0]
    return q, sc


def test_pack_layout(torch_cuda):
    """Packed tile layout: decoding every row gives back the planar input; pad rows stay zero."""
    from diolkos_b200 import ops

    rng = np.random.default_rng(3)
    for n, d in [(288, 5), (1056, 37), (4096, 70), (11008, 9), (4096, 4096 + 2 * 1024)]:
        q = rng.integers(-127, 128, n * d, dtype=np.int8)
        s = rng.standard_normal(n * d // 32).astype(np.float32)
        w = ops.pack(_dev(torch_cuda, q), _dev(torch_cuda, s), n, d).cpu().numpy()
        T = ops.tile_rows(d)
        assert 1 <= T <= 32 and ops.row_bytes(n) == _row_bytes(n)
        tiles = (d + T - 1) // T
        assert w.size == tiles * T * _row_bytes(n) == ops.packed_bytes(n, d)
        rows = d if d < 300 else 300  # decode a prefix of the large case (pure-Python loops)
        gq, gs = _unpack(w, n, rows, T)
        np.testing.assert_array_equal(gq, q.reshape(d, n)[:rows])
        np.testing.assert_array_equal(gs, s.reshape(d, n // 32)[:rows])
        if tiles * T > d:  # the ragged last tile's pad rows are zero
            t = tiles - 1
            for r in range(d - t * T, T):
                for b in range((n + 511) // 512):
                    wb = min(512, n - 512 * b)
                    bb = (wb + wb // 8 + 15) // 16 * 16
                    off = t * T * _row_bytes(n) + T * 576 * b + r * bb
                    assert not w[off:off + bb].any()


@pytest.mark.parametrize("case", G.GEMV_CASES)
def test_gemv_bit_exact_golden(torch_cuda, kgold, case):
    """Weights quantised on the GPU, packed, GEMV on the GPU: output bits == the reference's."""
    from diolkos_b200 import ops

    n, d, seed = case
    wb, x = G.gemv_inputs(n, d, seed)
    q, s = ops.quantize_bf16(_dev(torch_cuda, wb.view(np.int16)))
    w = ops.pack(q, s, n, d)
    out = ops.matmul(_dev(torch_cuda, x), w, n, d).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), kgold[f"gemv_{n}x{d}"].view(np.uint32))


@pytest.mark.parametrize("shape", [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 32000)])
def test_gemv_full_shapes_bit_exact(torch_cuda, port, shape):
    """The four GEMV shapes of the benchmark ([out x in] = 4096x4096, 11008x4096, 4096x11008,
    32000x4096), seeded N(0,0.02) weights and N(0,1) input: GPU output bits == oracle's."""
    from diolkos_b200 import ops

    torch = torch_cuda
    n, d = shape
    g = torch.Generator(device="cuda").manual_seed(n * 7 + d)
    wf = torch.randn(d * n, generator=g, device="cuda", dtype=torch.float32) * 0.02
    wb = wf.to(torch.bfloat16).view(torch.int16)
    q, s = ops.quantize_bf16(wb)
    pq, ps = port.quant_bf16(wb.cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(q.cpu().numpy(), pq)
    w = ops.pack(q, s, n, d)
    x = torch.randn(n, generator=g, device="cuda", dtype=torch.float32)
    out = ops.matmul(x, w, n, d).cpu().numpy()
    np.testing.assert_array_equal(out.view(np.uint32), port.matmul(x.cpu().numpy(), pq, ps, n, d).view(np.uint32))
    # the pre-quantised entry point gives the same bits
    xq, xs = ops.quantize_f32(x)
    out2 = ops.matmul_q(xq, xs, w, n, d).cpu().numpy()
    np.testing.assert_array_equal(out2.view(np.uint32), out.view(np.uint32))


def test_gemv_repeatable_and_ragged(torch_cuda, port):
    """Shapes that do not divide the stage size or the SM count; repeated calls give the same bits."""
    from diolkos_b200 import ops

    torch = torch_cuda
    rng = np.random.default_rng(4)
    for n, d in [(32, 1), (64, 149), (96, 297), (8192, 1001), (28672, 40)]:
        wq = rng.integers(-127, 128, n * d, dtype=np.int8)
        ws = (rng.random(n * d // 32, dtype=np.float32) * 0.001).astype(np.float32)
        x = rng.standard_normal(n).astype(np.float32)
        w = ops.pack(_dev(torch, wq), _dev(torch, ws), n, d)
        a = ops.matmul(_dev(torch, x), w, n, d).cpu().numpy()
        b = ops.matmul(_dev(torch, x), w, n, d).cpu().numpy()
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
        np.testing.assert_array_equal(a.view(np.uint32), port.matmul(x, wq, ws, n, d).view(np.uint32))


def test_rmsnorm(torch_cuda, port):
    from diolkos_b200 import ops

    rng = np.random.default_rng(5)
    for n in (288, 4096, 8192):
        x = rng.standard_normal(n).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        got = ops.rmsnorm(_dev(torch_cuda, x), _dev(torch_cuda, w)).cpu().numpy()
        np.testing.assert_allclose(got, port.rmsnorm(x, w), rtol=1e-6, atol=1e-7)


def test_dequant(torch_cuda, port):
    from diolkos_b200 import ops

    rng = np.random.default_rng(6)
    q = rng.integers(-127, 128, 4096, dtype=np.int8)
    s = rng.standard_normal(128).astype(np.float32)
    got = ops.dequantize(_dev(torch_cuda, q), _dev(torch_cuda, s)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), port.dequant(q, s).view(np.uint32))


def _rope_table(seq_len, hs):
    """(cos, sin) of p * 1/10000^(2j/hs) in float32, [seq_len][hs/2][2] (src/transformer.c:90-95)."""
    j = np.arange(hs // 2, dtype=np.float32)
    freq = (np.float32(1.0) / np.power(np.float32(10000.0), (2 * j) / np.float32(hs))).astype(np.float32)
    val = (np.arange(seq_len, dtype=np.float32)[:, None] * freq[None, :]).astype(np.float32)
    return np.stack([np.cos(val), np.sin(val)], axis=-1).astype(np.float32)


def _attention_ref(qkv, rope, kc, vc, pos, H, KVH, hs):
    """float64 restatement of src/transformer.c:87-193 on a cache already holding 0..pos-1."""
    dim, kvd, half = H * hs, KVH * hs, hs // 2
    c, s = rope[pos, :, 0].astype(np.float64), rope[pos, :, 1].astype(np.float64)
    def rot(v):
        v = v.astype(np.float64).reshape(-1, hs)
        a, b = v[:, :half], v[:, half:]
        return np.concatenate([a * c - b * s, a * s + b * c], axis=1)
    q = rot(qkv[:dim])
    k = rot(qkv[dim:dim + kvd])
    v = qkv[dim + kvd:].astype(np.float64).reshape(KVH, hs)
    K = kc.astype(np.float64).copy()
    V = vc.astype(np.float64).copy()
    K[:, pos], V[:, pos] = k, v
    out = np.empty((H, hs))
    for h in range(H):
        g = h // (H // KVH)
        sc = K[g, :pos + 1] @ q[h] / np.sqrt(hs)
        e = np.exp(sc - sc.max())
        out[h] = (e / e.sum()) @ V[g, :pos + 1]
    return out.reshape(-1)


@pytest.mark.parametrize("H,KVH,hs,seq,pos", [(32, 32, 128, 4096, 0), (32, 32, 128, 4096, 1000),
                                              (8, 1, 64, 512, 300), (6, 6, 48, 256, 63)])
def test_attention_decode_vs_fp64(torch_cuda, H, KVH, hs, seq, pos):
    """dk_attention_decode (fp32 cache) against a float64 numpy attention, 1e-5 relative; the cache
    row at pos holds the rotated k and v afterwards."""
    from diolkos_b200 import ops

    torch = torch_cuda
    rng = np.random.default_rng(H * 1000 + pos)
    qkv = rng.standard_normal((H + 2 * KVH) * hs).astype(np.float32)
    kc = np.zeros((KVH, seq, hs), np.float32)
    vc = np.zeros((KVH, seq, hs), np.float32)
    kc[:, :pos] = rng.standard_normal((KVH, pos, hs))
    vc[:, :pos] = rng.standard_normal((KVH, pos, hs))
    rope = _rope_table(seq, hs)
    dk, dv = _dev(torch, kc), _dev(torch, vc)
    work = torch.zeros(ops.attention_work_bytes(H, KVH, hs, seq), dtype=torch.uint8, device="cuda")
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    out = ops.attention_decode(_dev(torch, qkv), _dev(torch, rope), dk, dv, p, H, KVH, hs, seq, work).cpu().numpy()
    ref = _attention_ref(qkv, rope, kc, vc, pos, H, KVH, hs)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    np.testing.assert_array_equal(dv[:, pos].cpu().numpy(), qkv[(H + KVH) * hs:].reshape(KVH, hs))
    assert not work[ops.attention_work_bytes(H, KVH, hs, seq) - 256:].any()  # counters back at zero


def test_gemv_batch_equals_single(torch_cuda):
    """dk_matmul_q8_0_batch (back-to-back GEMVs, the later ones started early) gives the same bits as
    one dk_matmul_q8_0 call per matrix."""
    from diolkos_b200 import ops

    torch = torch_cuda
    rng = np.random.default_rng(7)
    n, d = 4096, 1000
    ws = []
    for _ in range(3):
        q = rng.integers(-127, 128, n * d, dtype=np.int8)
        s = (rng.random(n * d // 32, dtype=np.float32) * 0.001).astype(np.float32)
        ws.append(ops.pack(_dev(torch, q), _dev(torch, s), n, d))
    x = _dev(torch, rng.standard_normal(n).astype(np.float32))
    batch = [ws[0], ws[1], ws[2], ws[1], ws[0]]
    got = ops.matmul_batch(x, batch, n, d).cpu().numpy()
    for i, w in enumerate(batch):
        one = ops.matmul(x, w, n, d).cpu().numpy()
        np.testing.assert_array_equal(got[i].view(np.uint32), one.view(np.uint32))


@pytest.mark.parametrize("n,d,count", [(4096, 4096, 33), (4160, 1000, 70), (288, 96, 2), (512, 4096, 1)])
def test_gemv_batch_launches_bit_exact(torch_cuda, n, d, count):
    """The batch's launch structure: one launch per 32 matrices (count 33 and 70: a second and third
    launch that start early and wait only before their stores), two CTA groups taking alternate matrices
    (an odd count leaves the second group one short; count 1 runs one group), a partial last block
    (n = 4160), a tile range with fewer tiles than SMs (d = 96).  Every output row equals one
    dk_matmul_q8_0 call's, bit for bit, and nothing is written past the last matrix's rows."""
    from diolkos_b200 import ops

    torch = torch_cuda
    rng = np.random.default_rng(n + d + count)
    ws = []
    for _ in range(5):
        q = rng.integers(-127, 128, n * d, dtype=np.int8)
        s = (rng.random(n * d // 32, dtype=np.float32) * 0.001 + 1e-6).astype(np.float32)
        ws.append(ops.pack(_dev(torch, q), _dev(torch, s), n, d))
    x = _dev(torch, rng.standard_normal(n).astype(np.float32))
    idx = [int(i) for i in rng.integers(0, len(ws), count)]
    out = torch.full((count + 1, d), float("nan"), dtype=torch.float32, device="cuda")
    ops.matmul_batch(x, [ws[i] for i in idx], n, d, out[:count])
    got = out.cpu().numpy()
    singles = [ops.matmul(x, w, n, d).cpu().numpy() for w in ws]
    for i, k in enumerate(idx):
        np.testing.assert_array_equal(got[i].view(np.uint32), singles[k].view(np.uint32), err_msg=f"matrix {i}")
    assert np.isnan(got[count]).all()


# Tile heights on 148 SMs: d 4096 / 12288 -> 28, d 4736 -> 32 (the pipelined TMA form, n % 128 == 0);
# d 300 / 1001 -> 3 / 7 and n 288 -> the simple form.
@pytest.mark.parametrize("n,d,ntok", [(4096, 4096, 32), (4096, 4096, 5), (11008, 4096, 37), (288, 864, 70),
                                      (4096, 300, 1), (8192, 1001, 33), (2048, 4736, 65), (4096, 12288, 130)])
def test_tensor_core_matmul_tokens_bit_exact(torch_cuda, port, n, d, ntok):
    """dk_matmul_q8_0_tokens (tcgen05 kind::i8, one MMA per 32-value group): every token's output row
    equals the GEMV on that token bit for bit (and so the oracle's), for shapes that leave partial
    M tiles, partial token tiles and a partial last 512-column block; and the accumulate form adds."""
    from diolkos_b200 import ops

    torch = torch_cuda
    rng = np.random.default_rng(n + d + ntok)
    wq = rng.integers(-127, 128, n * d, dtype=np.int8)
    ws = (rng.random(n * d // 32, dtype=np.float32) * 0.001 + 1e-5).astype(np.float32)
    w = ops.pack(_dev(torch, wq), _dev(torch, ws), n, d)
    x = torch.from_numpy(rng.standard_normal((ntok, n)).astype(np.float32)).cuda()
    xq = torch.empty((ntok, n), dtype=torch.int8, device="cuda")
    xs = torch.empty((ntok, n // 32), dtype=torch.float32, device="cuda")
    for t in range(ntok):
        q, s = ops.quantize_f32(x[t].contiguous())
        xq[t] = q
        xs[t] = s
    out = ops.matmul_tokens(xq, xs, w, n, d).cpu().numpy()
    for t in range(ntok):
        ref = ops.matmul_q(xq[t].contiguous(), xs[t].contiguous(), w, n, d).cpu().numpy()
        np.testing.assert_array_equal(out[t].view(np.uint32), ref.view(np.uint32), err_msg=f"token {t}")
    np.testing.assert_array_equal(
        out[0].view(np.uint32),
        port.matmul_q(xq[0].cpu().numpy(), xs[0].cpu().numpy(), wq, ws, n, d).view(np.uint32))
    base = torch.from_numpy(rng.standard_normal((ntok, d)).astype(np.float32)).cuda()
    acc = ops.matmul_tokens(xq, xs, w, n, d, out=base.clone(), accumulate=True).cpu().numpy()
    want = (torch.from_numpy(out).cuda() + base).cpu().numpy()  # fp32 adds, round to nearest
    np.testing.assert_array_equal(acc.view(np.uint32), want.view(np.uint32))
