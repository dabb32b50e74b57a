"""CPU oracle for sandmuon_b200 -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

A numpy restatement of SandMuon's eager FP32 reference path
(sandmuon/optimizer.py and sandmuon/coefficients.py of pxike/SandMuon).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU legs (cpu_baseline and
--impl reference) may import it, and only as the checker / the timed CPU
baseline.  The product (sandmuon_b200/) never imports it.

Pinning: tests/test_oracle_golden.py checks every function here against
golden vectors that tests/golden/make_golden.py produced by running the
reference package itself (fixtures committed under tests/golden/).

Arithmetic is float32 like the reference, with float64 only where noted.
Matrix products go through numpy's BLAS (multithreaded), so the oracle's cost
is comparable to the reference's torch CPU path.
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32
TINY = np.finfo(np.float32).tiny

# sandmuon/coefficients.py:3-10
S8_MARGIN = 1.35
S8_MULTIPLIER = 1.0
S8_COEFFICIENTS = (
    (11.062126275847973, -56.051653229128085, 72.32081107619855),
    (4.100720073616268, -2.9324183165353577, 0.5339692084282731),
    (3.930310192522361, -2.873509793709714, 0.5366557527206212),
    (3.280567968245866, -2.414925589994015, 0.48635134757825227),
    (2.282741575232451, -1.6302296637355072, 0.40275720810675486),
)
STATISTIC_BETA = 0.97   # sandmuon/optimizer.py:123
MOMENTUM = 0.8          # sandmuon/optimizer.py:139
ADAMW = dict(lr_ratio=0.1, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)  # :139-143


def _f(x):
    return np.asarray(x, dtype=F32)


# ----------------------------------------------------------------- whiteners

def diagonal_inverse_sqrt(value):
    """sandmuon/optimizer.py:19-24."""
    value = _f(value)
    mean = F32(value.mean(dtype=F32))
    normalized = np.maximum(value, F32(mean * F32(1e-6))) / max(mean, TINY)
    return (F32(1.0) / np.sqrt(np.maximum(normalized, F32(1e-6)))).astype(F32)


def rank1_inverse_sqrt(second, mean):
    """sandmuon/optimizer.py:27-35 -> (inverse, z, coefficient)."""
    second, mean = _f(second), _f(mean)
    scale = max(F32(second.mean(dtype=F32)), TINY)
    variance = np.maximum(second - mean * mean, F32(0.0))
    inverse = (F32(1.0) / np.sqrt(np.maximum(variance / scale, F32(1e-6)))).astype(F32)
    z = (inverse * (mean / np.sqrt(F32(scale)))).astype(F32)
    root = F32(np.sqrt(F32(1.0) + F32((z * z).sum(dtype=F32))))
    coefficient = F32(-1.0) / (root * (root + F32(1.0)))
    return inverse, z, F32(coefficient)


def rank1_whiten(matrix, left, right):
    """sandmuon/optimizer.py:38-45, batched over the leading axis."""
    li, lz, lc = left
    ri, rz, rc = right
    lc = np.asarray(lc, F32).reshape(np.shape(lc) + (1, 1))
    rc = np.asarray(rc, F32).reshape(np.shape(rc) + (1, 1))
    v = _f(matrix) * _f(li)[..., :, None] * _f(ri)[..., None, :]
    v = v + lc * _f(lz)[..., :, None] * np.matmul(_f(lz)[..., None, :], v)
    v = v + rc * np.matmul(v, _f(rz)[..., :, None]) * _f(rz)[..., None, :]
    return v.astype(F32)


def rank1_mapback(value, left, right):
    """sandmuon/optimizer.py:48-60 (rank-one actions, then the diagonals)."""
    li, lz, lc = left
    ri, rz, rc = right
    v = _f(value)
    v = v + F32(lc) * _f(lz)[:, None] * (_f(lz)[None, :] @ v)
    v = v + F32(rc) * (v @ _f(rz)[:, None]) * _f(rz)[None, :]
    return (v * _f(li)[:, None] * _f(ri)[None, :]).astype(F32)


def graft_direction(value, output_rows):
    """sandmuon/optimizer.py:63-66."""
    v = _f(value)
    norm = max(F32(np.sqrt(np.float64((v.astype(np.float64) ** 2).sum()))), TINY)
    return (v * F32(math.sqrt(float(output_rows)) / norm)).astype(F32)


# ---------------------------------------------------- one-sided (split_sides)
# The historical optimizer's split_sides option
# (reproduction/odl/optim/diagonal_weighted_pe.py:408-410, 500-543): only the
# activation side carries a rank-one factor (the cotangent side's z is zero),
# so the whitening and the finish apply the rank-one action on that side
# alone -- the left side for a transposed matrix, else the right.

def one_side_whiten(sources, left_inverse, right_inverse, z, coefficient, rank_one_left):
    """reproduction/odl/optim/diagonal_weighted_pe.py:141-148, batched."""
    c = np.asarray(coefficient, F32).reshape(-1, 1, 1)
    v = (_f(sources) * _f(left_inverse)[:, :, None] * _f(right_inverse)[:, None, :]).astype(F32)
    if rank_one_left:
        return (v + c * _f(z)[:, :, None] * np.matmul(_f(z)[:, None, :], v)).astype(F32)
    return (v + c * np.matmul(v, _f(z)[:, :, None]) * _f(z)[:, None, :]).astype(F32)


def one_side_finish(q, left_inverse, right_inverse, z, coefficient, rank_one_left, q_scale, graft_rows):
    """reproduction/odl/optim/diagonal_weighted_pe.py:152-164, batched: the
    one-sided mapback, then the graft to norm sqrt(rows) (which cancels the
    historical aspect factor q_scale)."""
    c = np.asarray(coefficient, F32).reshape(-1, 1, 1)
    v = (_f(q) * np.asarray(q_scale, F32).reshape(-1, 1, 1)).astype(F32)
    if rank_one_left:
        v = v + c * _f(z)[:, :, None] * np.matmul(_f(z)[:, None, :], v)
    else:
        v = v + c * np.matmul(v, _f(z)[:, :, None]) * _f(z)[:, None, :]
    v = (v * _f(left_inverse)[:, :, None] * _f(right_inverse)[:, None, :]).astype(F32)
    norms = np.sqrt((v.astype(np.float64) ** 2).sum(axis=(-2, -1), keepdims=True)).astype(F32)
    rows = np.sqrt(np.asarray(graft_rows, F32)).reshape(-1, 1, 1)
    return (v * (rows / np.maximum(norms, TINY))).astype(F32)


# ------------------------------------------------------------------------ S8

def s8_fp32(x):
    """sandmuon/optimizer.py:69-93 on a [batch, rows, cols] (or 2-D) array.

    Keeps the reference's batch-level zero test (`count_nonzero` over the
    whole batch, :75-76)."""
    x = _f(x)
    squeeze = x.ndim == 2
    if squeeze:
        x = x[None]
    transposed = x.shape[-2] > x.shape[-1]
    if transposed:
        x = np.swapaxes(x, -1, -2)
    if not np.count_nonzero(x):
        out = np.zeros_like(x)
    else:
        norm = np.sqrt((x.astype(np.float64) ** 2).sum(axis=(-2, -1), keepdims=True)).astype(F32)
        x = x / np.maximum(norm, F32(1e-30))
        gram = np.matmul(x, np.swapaxes(x, -1, -2))
        gram2 = np.matmul(gram, gram)
        g2n = np.sqrt((gram2.astype(np.float64) ** 2).sum(axis=(-2, -1), keepdims=True)).astype(F32)
        scale = np.maximum(F32(S8_MARGIN) * np.power(g2n, F32(0.25)), F32(1e-30)).astype(F32)
        eye = np.eye(x.shape[-2], dtype=F32)
        a, b, c = (F32(v) for v in S8_COEFFICIENTS[0])
        with np.errstate(divide="ignore", invalid="ignore"):
            p = a * eye + b * gram / (scale * scale) + c * gram2 / (scale ** 4)
            x = np.matmul(p, x) / scale
        for a, b, c in S8_COEFFICIENTS[1:]:
            gram = np.matmul(x, np.swapaxes(x, -1, -2))
            gram2 = np.matmul(gram, gram)
            p = F32(a) * eye + F32(b) * gram + F32(c) * gram2
            x = np.matmul(p, x)
        out = x * F32(S8_MULTIPLIER)
    if transposed:
        out = np.swapaxes(out, -1, -2)
    out = np.ascontiguousarray(out, dtype=F32)
    return out[0] if squeeze else out


# ---------------------------------------------------------------- statistics

def column_stats(rows, with_first):
    """Forward / cotangent hook reductions (sandmuon/optimizer.py:156-178):
    (sum of squares, sum) over rows of float32(rows); float64 accumulation."""
    r = np.asarray(rows, dtype=F32).astype(np.float64)
    sq = (r * r).sum(axis=0).astype(F32)
    first = r.sum(axis=0).astype(F32) if with_first else None
    return sq, first


def _ema(old, new, beta):
    # tensor.mul_(beta).add_(new, alpha=1-beta)
    return (old * F32(beta) + F32(1.0 - beta) * new).astype(F32)


# ----------------------------------------------------------------- optimizer

class OracleSandMuon:
    """State machine of DiagonalWeightedPE / RankOneAWeightedPE
    (sandmuon/optimizer.py:96-328) over named numpy arrays.

    matrices: ordered {name: (d_out, d_in)}; a_source: {name: source name}
    (q/k/v sharing already resolved); auxiliaries: ordered {name: shape}.
    Statistics are injected with add_a / add_b (the hook reductions)."""

    def __init__(self, matrices, a_source, auxiliaries=(), *, rank_one_a, lr, split_sides=False):
        self.split_sides = bool(split_sides) and bool(rank_one_a)
        self.matrices = dict(matrices)
        self.a_source = dict(a_source)
        self.auxiliaries = list(auxiliaries)
        self.rank_one_a = bool(rank_one_a)
        self.lr = float(lr)
        self.state: dict[str, dict] = {name: {} for name in list(self.matrices) + self.auxiliaries}

    # hooks (sandmuon/optimizer.py:151-179)
    def add_a(self, name, rows):
        st = self.state[name]
        sq, first = column_stats(rows, self.rank_one_a)
        if "a_sum" not in st:
            st["a_sum"] = np.zeros(sq.shape, F32)
            st["a_count"] = 0
            if self.rank_one_a:
                st["a_first_sum"] = np.zeros(sq.shape, F32)
        st["a_sum"] = (st["a_sum"] + sq).astype(F32)
        if self.rank_one_a:
            st["a_first_sum"] = (st["a_first_sum"] + first).astype(F32)
        st["a_count"] += len(rows)

    def add_b(self, name, rows):
        st = self.state[name]
        sq, _ = column_stats(rows, False)
        if "b_sum" not in st:
            st["b_sum"] = np.zeros(sq.shape, F32)
            st["b_count"] = 0
        st["b_sum"] = (st["b_sum"] + sq).astype(F32)
        st["b_count"] += len(rows)

    def inject(self, name, *, a_sum=None, a_first_sum=None, a_count=None, b_sum=None, b_count=None):
        """Writes accumulated sums directly (the step-only benchmark path)."""
        st = self.state[name]
        if a_sum is not None:
            st["a_sum"], st["a_count"] = _f(a_sum).copy(), int(a_count)
            if self.rank_one_a:
                st["a_first_sum"] = _f(a_first_sum).copy()
        if b_sum is not None:
            st["b_sum"], st["b_count"] = _f(b_sum).copy(), int(b_count)

    # sandmuon/optimizer.py:182-207
    def _finish_a(self, name):
        st = self.state[name]
        if st.get("a_count", 0) < 1:
            raise RuntimeError(f"Missing activation statistics: {name}")
        count = st["a_count"]
        second = (st["a_sum"] / F32(count)).astype(F32)
        if self.rank_one_a:
            mean = (st["a_first_sum"] / F32(count)).astype(F32)
            if "a_ema" not in st:
                st["a_ema"], st["a_mean_ema"] = second.copy(), mean.copy()
            else:
                st["a_ema"] = _ema(st["a_ema"], second, STATISTIC_BETA)
                st["a_mean_ema"] = _ema(st["a_mean_ema"], mean, STATISTIC_BETA)
            factor = rank1_inverse_sqrt(st["a_ema"], st["a_mean_ema"])
            st["a_first_sum"] = np.zeros_like(st["a_first_sum"])
        else:
            st["a_ema"] = second.copy() if "a_ema" not in st else _ema(st["a_ema"], second, STATISTIC_BETA)
            factor = diagonal_inverse_sqrt(st["a_ema"])
        st["a_sum"] = np.zeros_like(st["a_sum"])
        st["a_count"] = 0
        return factor, count

    # sandmuon/optimizer.py:209-222
    def _finish_b(self, name, expected):
        st = self.state[name]
        if st.get("b_count", 0) != expected:
            raise RuntimeError(f"Missing or mismatched cotangent statistics: {name}")
        b = (st["b_sum"] / F32(expected)).astype(F32)
        b = (b / max(F32(b.mean(dtype=F32)), TINY)).astype(F32)
        st["b_ema"] = b.copy() if "b_ema" not in st else _ema(st["b_ema"], b, STATISTIC_BETA)
        inverse = diagonal_inverse_sqrt(st["b_ema"])
        st["b_sum"] = np.zeros_like(st["b_sum"])
        st["b_count"] = 0
        return inverse

    def step(self, weights, grads, directions_out=None):
        """One optimizer step (sandmuon/optimizer.py:224-316); updates
        `weights` (dict of float32 arrays) in place.  Names missing from
        `grads` are skipped like parameters whose .grad is None."""
        items, a_cache = [], {}
        for name in self.matrices:
            if name not in grads:
                continue
            source = self.a_source[name]
            if source not in a_cache:
                a_cache[source] = self._finish_a(source)
            a_factor, count = a_cache[source]
            inv_b = self._finish_b(name, count)
            st = self.state[name]
            g = _f(grads[name])
            if "momentum_buffer" not in st:
                st["momentum_buffer"] = np.zeros_like(g)
            st["momentum_buffer"] = (st["momentum_buffer"] * F32(MOMENTUM) + F32(1 - MOMENTUM) * g).astype(F32)
            src = (st["momentum_buffer"] * F32(MOMENTUM) + g * F32(1 - MOMENTUM)).astype(F32)
            rows, cols = g.shape
            transposed = rows > cols
            zero = (np.zeros_like(inv_b), np.zeros_like(inv_b), F32(0.0))
            if transposed:
                src = src.T
                left, right = (a_factor, (inv_b, zero[1], zero[2])) if self.rank_one_a else (a_factor, inv_b)
            else:
                left, right = ((inv_b, zero[1], zero[2]), a_factor) if self.rank_one_a else (inv_b, a_factor)
            items.append((name, np.ascontiguousarray(src), left, right, transposed))

        for name in self.auxiliaries:
            if name in grads:
                self._adamw(name, weights, _f(grads[name]))

        groups: dict[tuple, list] = {}
        for item in items:
            groups.setdefault(item[1].shape, []).append(item)
        if self.split_sides:
            for entries in groups.values():
                self._step_one_sided(entries, weights, directions_out)
            return
        for entries in groups.values():
            sources = np.stack([e[1] for e in entries])
            if self.rank_one_a:
                li = np.stack([e[2][0] for e in entries]); lz = np.stack([e[2][1] for e in entries])
                lc = np.array([e[2][2] for e in entries], F32)
                ri = np.stack([e[3][0] for e in entries]); rz = np.stack([e[3][1] for e in entries])
                rc = np.array([e[3][2] for e in entries], F32)
                whitened = rank1_whiten(sources, (li, lz, lc), (ri, rz, rc))
            else:
                li = np.stack([e[2] for e in entries]); ri = np.stack([e[3] for e in entries])
                whitened = (sources * li[:, :, None] * ri[:, None, :]).astype(F32)
            q = s8_fp32(whitened)
            for index, (name, _, _, _, transposed) in enumerate(entries):
                if self.rank_one_a:
                    value = rank1_mapback(q[index], (li[index], lz[index], lc[index]),
                                          (ri[index], rz[index], rc[index]))
                else:
                    value = (q[index] * li[index][:, None] * ri[index][None, :]).astype(F32)
                direction = graft_direction(value, self.matrices[name][0])
                if transposed:
                    direction = direction.T
                if directions_out is not None:
                    directions_out[name] = np.ascontiguousarray(direction)
                weights[name] = (weights[name] + F32(-self.lr) * direction).astype(F32)

    def _step_one_sided(self, entries, weights, directions_out):
        """One shape group with split_sides (diagonal_weighted_pe.py:500-543):
        transposed matrices first (rank-one action on the left), then the
        others (on the right)."""
        entries = sorted(entries, key=lambda e: e[4], reverse=True)
        boundary = sum(1 for e in entries if e[4])
        # rank-one factors: (inverse, z, coefficient) of the A side; the B side's
        # (inverse, zero, zero) contributes its inverse only
        li = np.stack([e[2][0] for e in entries]); ri = np.stack([e[3][0] for e in entries])
        sources = np.stack([e[1] for e in entries])
        rows = np.array([self.matrices[e[0]][0] for e in entries], F32)
        cols = np.array([self.matrices[e[0]][1] for e in entries], F32)
        q_scale = np.sqrt(np.maximum(F32(1.0), rows / cols)).astype(F32)
        # pieces (first, end, rank-one on the left, z, coefficient); the z of the
        # two pieces differ in length (d_in on either side)
        pieces = []
        for lo, hi, left in ((0, boundary, True), (boundary, len(entries), False)):
            if hi > lo:
                side = 2 if left else 3
                pieces.append((lo, hi, left, np.stack([e[side][1] for e in entries[lo:hi]]),
                               np.array([e[side][2] for e in entries[lo:hi]], F32)))
        q = s8_fp32(np.concatenate([one_side_whiten(sources[lo:hi], li[lo:hi], ri[lo:hi], z, c, left)
                                    for lo, hi, left, z, c in pieces]))
        finished = [one_side_finish(q[lo:hi], li[lo:hi], ri[lo:hi], z, c, left, q_scale[lo:hi], rows[lo:hi])
                    for lo, hi, left, z, c in pieces]
        directions = np.concatenate(finished)
        for index, (name, _, _, _, transposed) in enumerate(entries):
            direction = directions[index].T if transposed else directions[index]
            if directions_out is not None:
                directions_out[name] = np.ascontiguousarray(direction)
            weights[name] = (weights[name] + F32(-self.lr) * direction).astype(F32)

    # sandmuon/optimizer.py:268-281
    def _adamw(self, name, weights, g):
        st = self.state[name]
        if "exp_avg" not in st:
            st["exp_avg"] = np.zeros_like(g)
            st["exp_avg_sq"] = np.zeros_like(g)
            st["step"] = 0
        st["step"] += 1
        b1, b2 = ADAMW["betas"]
        st["exp_avg"] = (st["exp_avg"] * F32(b1) + F32(1 - b1) * g).astype(F32)
        st["exp_avg_sq"] = (st["exp_avg_sq"] * F32(b2) + F32(1 - b2) * g * g).astype(F32)
        bias1, bias2 = 1 - b1 ** st["step"], 1 - b2 ** st["step"]
        update = (st["exp_avg"] / F32(bias1)) / (np.sqrt(st["exp_avg_sq"] / F32(bias2)) + F32(ADAMW["eps"]))
        lr = self.lr * ADAMW["lr_ratio"]
        weights[name] = (weights[name] * F32(1 - lr * ADAMW["weight_decay"])).astype(F32)
        weights[name] = (weights[name] + F32(-lr) * update.astype(F32)).astype(F32)
