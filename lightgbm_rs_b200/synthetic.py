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


def mixed_c3(num_data=2_000_000, seed=0, chunk=1 << 18):
    """C3 categorical + NaN regression stand-in.

    90 numeric features ~ N(0,1) with 10 % NaN (Bernoulli mask); 10 categorical features
    with cardinalities spread evenly over 16..240 and Zipf(1.2) codes (clipped to the
    cardinality); y = sum of 10 depth-3 step functions (3 random features each,
    thresholds at random sample quantiles, 8 leaf values ~ N(0,1); NaN goes right) +
    N(0,1). Cardinalities stop at 240 so every categorical feature keeps at most 256
    bins after the reference's 99 % category cut. Returns X (f64, categorical columns
    last), y, and the categorical column indices."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n_num, n_cat = 90, 10
    cards = np.linspace(16, 240, n_cat).astype(np.int64)
    F = n_num + n_cat
    X = np.empty((num_data, F), dtype=np.float64)
    for r0 in range(0, num_data, chunk):
        r1 = min(num_data, r0 + chunk)
        x = rng.standard_normal((r1 - r0, n_num))
        x[rng.random((r1 - r0, n_num)) < 0.1] = np.nan
        X[r0:r1, :n_num] = x
        for j in range(n_cat):
            X[r0:r1, n_num + j] = np.minimum(rng.zipf(1.2, r1 - r0) - 1, cards[j] - 1)
    sample = X[rng.choice(num_data, min(num_data, 20000), replace=False)]
    y = rng.standard_normal(num_data)
    for _ in range(10):
        feats = rng.choice(F, 3, replace=False)
        thr = [np.nanquantile(sample[:, f], rng.uniform(0.2, 0.8)) for f in feats]
        leaves = rng.standard_normal(8)
        idx = np.zeros(num_data, dtype=np.int64)
        for k, (f, t) in enumerate(zip(feats, thr)):
            idx |= (np.nan_to_num(X[:, f], nan=np.inf) > t).astype(np.int64) << k
        y += leaves[idx]
    return X, y.astype(np.float32), list(range(n_num, F))


def rank_c4(num_queries=20_000, num_features=700, seed=0):
    """C4 lambdarank stand-in.

    Query sizes ~ Poisson(23) clipped to [1, 200] (about 473k rows); 700 features, 80 %
    exactly 0, else Exp(1); relevance 0..4 drawn from a softmax over the distances of a
    random linear score to 5 thresholds at its 20/40/60/80/95 % quantiles. Returns X
    (f32), labels (f32), query sizes."""
    rng = np.random.Generator(np.random.PCG64(seed))
    sizes = np.clip(rng.poisson(23, num_queries), 1, 200)
    n = int(sizes.sum())
    X = np.zeros((n, num_features), dtype=np.float32)
    chunk = 1 << 15
    for r0 in range(0, n, chunk):
        r1 = min(n, r0 + chunk)
        m = rng.random((r1 - r0, num_features)) < 0.2
        X[r0:r1][m] = rng.exponential(1.0, int(m.sum())).astype(np.float32)
    w = rng.standard_normal(num_features)
    z = X.astype(np.float64) @ w
    z = (z - z.mean()) / (z.std() + 1e-12)
    t = np.quantile(z, [0.2, 0.4, 0.6, 0.8, 0.95])
    logits = -np.abs(z[:, None] - t[None, :]) * 3.0
    p = np.exp(logits - logits.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    u = rng.random(n)
    y = (u[:, None] > np.cumsum(p, axis=1)).sum(axis=1).clip(0, 4).astype(np.float32)
    return X, y, sizes
