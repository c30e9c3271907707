"""Host-side inputs of one training sample (the small CPU parts of the reference's step).

expo_features  src/sa3_pipeline.h:57-67  [cos, sin](2 pi t f), f log-spaced in [min_f, max_f]
sample_at      src/train_diffusion.h:62-78  x_t = (1 - t) z + t n,  v = n - z
Both restate the reference's float32 arithmetic in numpy (the device step consumes the results).
"""
import math

import numpy as np


def expo_features(t, dim, min_f, max_f):
    half = dim // 2
    lmin = np.float32(math.log(min_f))
    lmax = np.float32(math.log(max_f))
    i = np.arange(half, dtype=np.float32)
    ramp = i / np.float32(half - 1) if half > 1 else np.zeros(half, np.float32)
    freq = np.exp((ramp * (lmax - lmin) + lmin).astype(np.float32)).astype(np.float32)
    arg = (np.float32(t) * freq * np.float32(6.28318530717958648)).astype(np.float32)
    return np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)


def sample_at(z, t, noise):
    """(x_t, velocity target) for latent z, timestep t and a given noise draw (float32)."""
    z = np.asarray(z, np.float32)
    n = np.asarray(noise, np.float32)
    t = np.float32(t)
    return ((np.float32(1.0) - t) * z + t * n).astype(np.float32), (n - z).astype(np.float32)
