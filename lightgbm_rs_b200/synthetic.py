"""Seeded synthetic stand-ins for the benchmark configurations.

No public dataset is named for these configurations, so inputs are generated with
the stated shapes and distributions (numpy PCG64, fixed seeds):

  C0/C1 binary: X ~ N(0,1) f32 [N x 28]; x_0..x_6 <- exp(x); w ~ N(0,1)^28;
                y ~ Bernoulli(sigmoid(w.x + 0.5 x0 x1)) using the transformed x.
  C2 wide:      X ~ U(-1,1) f32 [N x 2000]; 50 random features j with v_j ~ N(0,1);
                y = 1[sum v_j x_j + N(0, 0.1^2) > 0].
"""

import numpy as np


def binary_c0(num_data=100_000, num_features=28, seed=0, chunk=1 << 20):
    """Rows are generated in chunks so 10.5M x 28 stays within a few GB."""
    rng = np.random.Generator(np.random.PCG64(seed))
    w = rng.standard_normal(num_features)
    X = np.empty((num_data, num_features), dtype=np.float32)
    y = np.empty(num_data, dtype=np.float32)
    for r0 in range(0, num_data, chunk):
        r1 = min(num_data, r0 + chunk)
        x = rng.standard_normal((r1 - r0, num_features)).astype(np.float32)
        x[:, :7] = np.exp(x[:, :7])
        z = x.astype(np.float64) @ w + 0.5 * x[:, 0].astype(np.float64) * x[:, 1]
        p = 1.0 / (1.0 + np.exp(-z))
        y[r0:r1] = (rng.random(r1 - r0) < p).astype(np.float32)
        X[r0:r1] = x
    return X, y


def wide_c2(num_data=400_000, num_features=2000, seed=0, chunk=1 << 16):
    rng = np.random.Generator(np.random.PCG64(seed))
    j = rng.choice(num_features, 50, replace=False)
    v = rng.standard_normal(50)
    X = np.empty((num_data, num_features), dtype=np.float32)
    y = np.empty(num_data, dtype=np.float32)
    for r0 in range(0, num_data, chunk):
        r1 = min(num_data, r0 + chunk)
        x = rng.uniform(-1.0, 1.0, (r1 - r0, num_features)).astype(np.float32)
        z = x[:, j].astype(np.float64) @ v + rng.normal(0.0, 0.1, r1 - r0)
        y[r0:r1] = (z > 0).astype(np.float32)
        X[r0:r1] = x
    return X, y
