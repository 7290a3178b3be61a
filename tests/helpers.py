"""Seeded input builders shared by the GPU parity tests."""
import numpy as np


def bf16_tensor(oracle, x):
    """fp32 numpy -> (torch bf16 CUDA tensor, the same values as fp32 numpy)."""
    import torch
    bits = oracle.f32_to_bf16_bits(np.ascontiguousarray(x, np.float32))
    t = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    return t, oracle.bf16_bits_to_f32(bits)


def f32_tensor(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def to_f32(t):
    import torch
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


def decode_case(rng, B, lens, H, Hkv, d, bs, num_blocks, max_blocks=None):
    """Random q/pools and block tables drawn from a seeded permutation of the pool."""
    lens = np.asarray(lens, np.int32)
    nblk = (lens + bs - 1) // bs
    mb = int(max_blocks or max(1, nblk.max()))
    assert nblk.sum() <= num_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    table = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        table[b, : nblk[b]] = perm[off: off + nblk[b]]
        off += nblk[b]
    q = rng.standard_normal((B, H, d)).astype(np.float32)
    kp = rng.standard_normal((num_blocks, Hkv, bs, d)).astype(np.float32)
    vp = rng.standard_normal((num_blocks, Hkv, bs, d)).astype(np.float32)
    return q, kp, vp, table, lens


def rel_err(got, ref):
    scale = max(float(np.max(np.abs(ref))), 1e-30)
    return float(np.max(np.abs(got - ref))) / scale
