"""dk_attention_decode_noalloc (static device scratch) against dk_attention_decode (caller scratch).

Collected last on purpose (file name): it must pass both on its own in a fresh process, where its
first call also does the per-device setup, and after every other test has run in the same process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20  # the static scratch the header states


def _rope_table(seq_len, hs):
    j = np.arange(hs // 2, dtype=np.float32)
    freq = (np.float32(1.0) / np.power(np.float32(10000.0), (2 * j) / np.float32(hs))).astype(np.float32)
    val = (np.arange(seq_len, dtype=np.float32)[:, None] * freq[None, :]).astype(np.float32)
    return np.stack([np.cos(val), np.sin(val)], axis=-1).astype(np.float32)


@pytest.fixture(scope="module")
def torch_cuda():
    import torch

    torch.cuda.init()
    return torch


# (n_heads, n_kv_heads, head_size, seq_len, cache dtype, the two positions called in a row)
CASES = [(32, 32, 128, 4096, "f32", (1000, 1001)),   # 7B shape, 16 splits per KV head
         (8, 1, 64, 512, "bf16", (300, 301)),        # GQA, truncating bf16 cache
         (64, 8, 128, 4096, "f32", (2047, 2048))]    # 70B-shape heads, largest scratch of the three


@pytest.mark.parametrize("H,KVH,hs,seq,kv,positions", CASES)
def test_noalloc_matches_regular_entry(torch_cuda, H, KVH, hs, seq, kv, positions):
    from diolkos_b200 import ops

    torch = torch_cuda
    need = ops.attention_work_bytes(H, KVH, hs, seq)
    assert 0 < need + 256 <= SCRATCH_BYTES
    rng = np.random.default_rng(H + seq)
    dt = torch.float32 if kv == "f32" else torch.int16
    p_hi = max(positions)
    kc0 = torch.zeros((KVH, seq, hs), dtype=torch.float32, device="cuda")
    vc0 = torch.zeros_like(kc0)
    kc0[:, :p_hi] = torch.from_numpy(rng.standard_normal((KVH, p_hi, hs)).astype(np.float32)).cuda()
    vc0[:, :p_hi] = torch.from_numpy(rng.standard_normal((KVH, p_hi, hs)).astype(np.float32)).cuda()
    if kv == "bf16":
        kc0 = kc0.to(torch.bfloat16).view(torch.int16)
        vc0 = vc0.to(torch.bfloat16).view(torch.int16)
    assert kc0.dtype == dt
    rope = torch.from_numpy(_rope_table(seq, hs)).cuda()
    qkvs = [torch.from_numpy(rng.standard_normal((H + 2 * KVH) * hs).astype(np.float32)).cuda() for _ in positions]
    pos = [torch.tensor([p], dtype=torch.int32, device="cuda") for p in positions]

    # regular entry: caller-provided, zero-filled scratch
    kc_a, vc_a = kc0.clone(), vc0.clone()
    work = torch.zeros(need, dtype=torch.uint8, device="cuda")
    outs_a = [torch.empty(H * hs, dtype=torch.float32, device="cuda") for _ in positions]
    # no-alloc entry: every buffer it touches besides its own static scratch is allocated up front
    kc_b, vc_b = kc0.clone(), vc0.clone()
    outs_b = [torch.empty(H * hs, dtype=torch.float32, device="cuda") for _ in positions]

    for i in range(len(positions)):
        ops.attention_decode(qkvs[i], rope, kc_a, vc_a, pos[i], H, KVH, hs, seq, work, out=outs_a[i])
    torch.cuda.synchronize()

    ops.attention_decode_noalloc(qkvs[0], rope, kc_b, vc_b, pos[0], H, KVH, hs, seq, outs_b[0])
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for i in range(1, len(positions)):
        ops.attention_decode_noalloc(qkvs[i], rope, kc_b, vc_b, pos[i], H, KVH, hs, seq, outs_b[i])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "device memory changed across a no-alloc call"

    for a, b in zip(outs_a, outs_b):
        assert torch.isfinite(a).all()
        np.testing.assert_array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(kc_a.cpu().numpy(), kc_b.cpu().numpy())
    np.testing.assert_array_equal(vc_a.cpu().numpy(), vc_b.cpu().numpy())


def test_noalloc_rejects_oversized_shape(torch_cuda):
    """A shape whose scratch exceeds the static array is refused before anything is launched."""
    from diolkos_b200 import _native, ops

    torch = torch_cuda
    H, KVH, hs, seq = 8192, 1024, 128, 64  # one split per KV head, 8192 * 130 fp32 partials > 4 MiB
    assert ops.attention_work_bytes(H, KVH, hs, seq) + 256 > SCRATCH_BYTES
    dummy = torch.zeros(64, dtype=torch.float32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(_native.DiolkosError) as ei:
        ops.attention_decode_noalloc(dummy, dummy, dummy, dummy, pos, H, KVH, hs, seq, dummy)
    assert ei.value.code == _native.DK_ERR_INVALID
    assert "static scratch" in str(ei.value)
