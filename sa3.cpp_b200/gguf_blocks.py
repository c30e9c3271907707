"""Synthetic frozen-base weights as GGUF Q8_0 / Q4_K / F16 / F32 row bytes (numpy).

The reference quantizes its checkpoints offline with tools/sa3-quantize.cpp (rows along ne[0] =
in, only when in % block == 0, tools/sa3-quantize.cpp:75-85); the benchmarks here need the same
kind of bytes for seeded synthetic weights.  Q8_0 follows the published GGUF rounding (d =
amax / 127, q = round-half-away(x / d)); Q4_K uses a simple per-sub-block affine fit, which is a
valid encoding (only decoding has to be exact, and decoding happens on the device).
"""
import numpy as np


def _round_half_away(x):
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def q8_0(w):
    w = np.ascontiguousarray(w, np.float32)
    out, inn = w.shape
    assert inn % 32 == 0
    b = w.reshape(out, inn // 32, 32)
    d = (np.abs(b).max(-1, keepdims=True) / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = _round_half_away((b * inv).astype(np.float32)).astype(np.int8)
    blk = np.empty((out, inn // 32, 34), np.uint8)
    blk[..., :2] = d.astype(np.float16).view(np.uint8).reshape(out, inn // 32, 2)
    blk[..., 2:] = q.view(np.uint8)
    return blk.reshape(out, -1)


def q4_k(w):
    w = np.ascontiguousarray(w, np.float32)
    out, inn = w.shape
    assert inn % 256 == 0
    nsb = inn // 256
    x = w.reshape(out, nsb, 8, 32)
    lo = np.minimum(x.min(-1), 0.0).astype(np.float32)
    hi = np.maximum(x.max(-1), lo).astype(np.float32)
    scale = (hi - lo) / np.float32(15)
    minv = -lo
    d = (scale.max(-1) / np.float32(63)).astype(np.float16)
    dmin = (minv.max(-1) / np.float32(63)).astype(np.float16)
    df = d.astype(np.float32)[..., None]
    mf = dmin.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.rint(scale / df), 0).clip(0, 63).astype(np.uint8)
        mn = np.where(mf > 0, np.rint(minv / mf), 0).clip(0, 63).astype(np.uint8)
        d1 = (df * sc.astype(np.float32))[..., None]
        m1 = (mf * mn.astype(np.float32))[..., None]
        q = np.where(d1 > 0, np.rint((x + m1) / d1), 0).clip(0, 15).astype(np.uint8)
    blk = np.zeros((out, nsb, 144), np.uint8)
    blk[..., 0:2] = d.view(np.uint8).reshape(out, nsb, 2)
    blk[..., 2:4] = dmin.view(np.uint8).reshape(out, nsb, 2)
    s12 = blk[..., 4:16]
    s12[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    s12[..., 4:8] = mn[..., 0:4] | ((mn[..., 4:8] >> 4) << 6)
    s12[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mn[..., 4:8] & 0x0F) << 4)
    # 4 chunks of 32 bytes: low nibble = sub-block 2j, high nibble = sub-block 2j+1
    qq = q.reshape(out, nsb, 4, 2, 32)
    blk[..., 16:] = (qq[:, :, :, 0, :] | (qq[:, :, :, 1, :] << 4)).reshape(out, nsb, 128)
    return blk.reshape(out, -1)


def encode(w, qtype):
    if qtype == "q8_0":
        return q8_0(w)
    if qtype == "q4_k":
        return q4_k(w)
    if qtype == "f16":
        w16 = np.ascontiguousarray(w, np.float16)
        return w16.view(np.uint8).reshape(w.shape[0], -1)
    if qtype == "f32":
        w32 = np.ascontiguousarray(w, np.float32)
        return w32.view(np.uint8).reshape(w.shape[0], -1)
    raise ValueError(qtype)


def q8_0_torch(w):
    """Q8_0 row bytes of a CUDA float32 tensor [out][in] (a valid encoding, built on the GPU so that
    billion-parameter synthetic checkpoints are quick to make); returns a host uint8 array."""
    import torch
    out, inn = w.shape
    assert inn % 32 == 0
    b = w.reshape(out, inn // 32, 32)
    d = (b.abs().amax(-1, keepdim=True) / 127.0).to(torch.float32)
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = torch.round(b * inv).clamp_(-127, 127).to(torch.int8)
    blk = torch.empty(out, inn // 32, 34, dtype=torch.uint8, device=w.device)
    blk[..., :2] = d.to(torch.float16).view(torch.uint8)
    blk[..., 2:] = q.view(torch.uint8)
    return blk.reshape(out, -1).cpu().numpy()
