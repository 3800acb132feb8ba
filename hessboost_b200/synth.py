"""Seeded synthetic inputs with the shapes and distributions of the
benchmark configurations (no public dataset is involved).

C1: regression, rows x 28 N(0,1), y = sin x0 + x1 x2 + 0.5 x3^2 - x4 + N(0, 0.1).
C2: binary logistic, rows x 28 N(0,1) with 5% of cells NaN (mask drawn
    after the values), y ~ Bernoulli(sigmoid(w . x~ + 0.3 x0 x1)),
    w ~ N(0,1)/sqrt(28), x~ = x with NaN -> 0.
C4: wide sparse binary, CSR rows x F with each cell stored with
    probability `density` (column positions uniform), values
    lognormal(0, 1), absent cells missing; 20 random features carry
    N(0, 1) weights and y ~ Bernoulli(sigmoid(sum of the weights of the
    row's stored features)).
C5: prediction, a forest of complete depth-d trees over F features with
    thresholds from N(0,1) quantiles, uniform default directions and
    N(0, 0.01) leaves; rows N(0,1) with 1% NaN.
"""

import numpy as np


def regression_c1(n_rows=1_000_000, n_cols=28, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_rows, n_cols), dtype=np.float32)
    x0, x1, x2, x3, x4 = (x[:, i].astype(np.float64) for i in range(5))
    y = np.sin(x0) + x1 * x2 + 0.5 * x3 * x3 - x4 + rng.normal(0.0, 0.1, n_rows)
    return x, y.astype(np.float32)


def logistic_c2(n_rows=10_000_000, n_cols=28, seed=0, missing=0.05):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_rows, n_cols), dtype=np.float32)
    mask = rng.random((n_rows, n_cols), dtype=np.float32) < missing
    w = rng.standard_normal(n_cols).astype(np.float32) / np.float32(np.sqrt(n_cols))
    xz = np.where(mask, np.float32(0.0), x)  # labelling treats NaN as 0
    logits = xz @ w + np.float32(0.3) * xz[:, 0] * xz[:, 1]
    del xz
    x[mask] = np.nan
    del mask
    p = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    y = (rng.random(n_rows) < p).astype(np.float32)
    return x, y


def multiclass_c3(n_rows=2_000_000, n_cols=100, n_classes=10, seed=0):
    """C3: U(-1, 1) features; the label is the argmax over n_classes random
    linear projections (weights N(0, 1)) plus Gumbel(0, 1) noise."""
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, (n_rows, n_cols)).astype(np.float32)
    w = rng.standard_normal((n_cols, n_classes)).astype(np.float32)
    y = np.empty(n_rows, np.float32)
    step = 1 << 20
    for a in range(0, n_rows, step):
        z = x[a:a + step] @ w + rng.gumbel(size=(min(step, n_rows - a), n_classes)).astype(np.float32)
        y[a:a + step] = np.argmax(z, axis=1)
    return x, y


def forest_c5(n_trees=1000, depth=8, n_cols=50, seed=0):
    """Complete trees as a node array (the library's hb_tree_node layout)."""
    from . import NODE_DTYPE

    rng = np.random.default_rng(seed)
    per = 2 ** (depth + 1) - 1
    nodes = np.zeros(n_trees * per, NODE_DTYPE)
    qs = np.sort(rng.standard_normal(4096)).astype(np.float32)
    for t in range(n_trees):
        a = nodes[t * per : (t + 1) * per]
        internal = 2**depth - 1
        idx = np.arange(per)
        a["left"] = np.where(idx < internal, 2 * idx + 1, -1)
        a["right"] = np.where(idx < internal, 2 * idx + 2, -1)
        a["split_feature"] = np.where(idx < internal, rng.integers(0, n_cols, per), 0)
        a["split_cond"] = np.where(idx < internal, qs[rng.integers(0, len(qs), per)], 0.0)
        a["default_left"] = np.where(idx < internal, rng.integers(0, 2, per), 1)
        a["leaf_value"] = np.where(idx < internal, 0.0, rng.normal(0.0, 0.01, per)).astype(np.float32)
        a["split_bin"] = -1
    tree_ptr = np.arange(n_trees + 1, dtype=np.uint64) * per
    return nodes, tree_ptr


def rows_c5(n_rows, n_cols=50, seed=1, missing=0.01):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_rows, n_cols), dtype=np.float32)
    x[rng.random((n_rows, n_cols), dtype=np.float32) < missing] = np.nan
    return x


def sparse_c4(n_rows=5_000_000, n_cols=2000, density=0.02, seed=0, n_weighted=20):
    """C4 as CSR arrays: (indptr u64, indices u32 ascending within a row,
    values f32, y f32). Each cell of the row-major n_rows x n_cols grid is
    stored independently with probability `density`: the gaps between
    stored cells are geometric."""
    rng = np.random.default_rng(seed)
    k = min(n_weighted, n_cols)
    w = np.zeros(n_cols, np.float64)
    w[rng.choice(n_cols, size=k, replace=False)] = rng.standard_normal(k)
    cells = n_rows * n_cols
    parts = []
    at = -1
    step = 1 << 24
    while True:
        pos = at + np.cumsum(rng.geometric(density, size=step).astype(np.int64))
        keep = pos[pos < cells]
        parts.append(keep)
        if keep.size < pos.size:
            break
        at = int(pos[-1])
    pos = np.concatenate(parts)
    del parts
    rows = pos // n_cols
    indices = (pos - rows * n_cols).astype(np.uint32)
    del pos
    indptr = np.zeros(n_rows + 1, np.uint64)
    np.cumsum(np.bincount(rows, minlength=n_rows), out=indptr[1:])
    logits = np.bincount(rows, weights=w[indices], minlength=n_rows)
    del rows
    values = rng.lognormal(0.0, 1.0, size=indices.size).astype(np.float32)
    y = (rng.random(n_rows) < 1.0 / (1.0 + np.exp(-logits))).astype(np.float32)
    return indptr, indices, values, y


def csr_to_dense(indptr, indices, values, n_cols):
    """The dense f32 matrix of CSR arrays, absent cells NaN."""
    n = len(indptr) - 1
    x = np.full((n, n_cols), np.nan, np.float32)
    rows = np.repeat(np.arange(n), np.diff(np.asarray(indptr, np.int64)))
    x[rows, np.asarray(indices, np.int64)] = values
    return x
