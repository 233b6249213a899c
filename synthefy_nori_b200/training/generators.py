"""The synthetic-table prior mixture: generator families and augmentations, on the device.

Families (behaviour of the reference's ``training/data_generator.py`` episodes; every
regression table is standardised with its context rows at the end):

* ``scm``              meta-sampled MLP / tree structural causal models (``scm_prior``);
* ``tree``             averaged random decision trees over mixed continuous /
                       categorical features (piecewise-constant targets);
* ``gp``               Gaussian-process functions by random Fourier features (RBF or
                       Matern spectral densities, per-feature length scales) on a few
                       correlated active features;
* ``quadratic``        ``x^T M x + w^T x + b`` (+ occasional cubic terms) on an active
                       subset with a spectrally scaled symmetric ``M``;
* ``sparse_nonlinear`` latent-factor feature blocks, a few strong predictors through
                       random nonlinear functions, weak linear background, threshold
                       regimes, heteroskedastic noise;
* ``lookup``           1-3 entity-ID columns with Zipf frequencies whose per-entity
                       effects drive the target, plus continuous signal;
* ``cat_dominant``     60-95 % categorical columns, per-level effects (nominal or
                       ordinal), pairwise category interactions;
* ``binary``           binary fingerprints (rare on-bits) with a sparse target;
* ``temporal``         rows in time order: AR(1) features, lagged targets, concept
                       drift, trend + seasonality;
* ``clean_lowdim``     5-30 mostly categorical features with simple rules, low noise.

Noise is calibrated so the context rows reach a sampled target R^2 (one scale factor
on a sampled noise shape).  Augmentations (per table, then per column): monotone shape
transforms (exp / log / power / rank / sign flip), numeric-to-categorical binning,
heavy-tailed spikes, and missingness (completely at random, or driven by another
column's tail).

B200 design: per-table choices are a handful of host draws; the data itself is built
with batched tensor ops on the table's device (tables of one family in one call), so a
step's batch never leaves the GPU.
"""

from __future__ import annotations

import math

import numpy as np
import torch

DEFAULT_FAMILY_PROBS = {"scm": 0.34, "tree": 0.08, "gp": 0.12, "quadratic": 0.06, "sparse_nonlinear": 0.08,
                        "lookup": 0.04, "cat_dominant": 0.08, "binary": 0.04, "temporal": 0.10, "clean_lowdim": 0.06}


# ------------------------------------------------------------------ helpers
def _standardize_cols(X, fit_rows):
    ref = X[:fit_rows]
    mu = ref.mean(0, keepdim=True)
    sd = ref.std(0, unbiased=False, keepdim=True)
    return torch.where(sd > 1e-8, (X - mu) / sd.clamp(min=1e-8), X - mu)


def _continuous(N, F, rng, gen, device):
    """Columns from a mix of normal, uniform(-2, 2), scaled beta and Student-t."""
    cols = []
    for _ in range(F):
        kind = int(rng.integers(0, 4))
        if kind == 0:
            c = torch.randn(N, generator=gen, device=device)
        elif kind == 1:
            c = torch.rand(N, generator=gen, device=device) * 4 - 2
        elif kind == 2:
            a, b = rng.uniform(0.5, 5.0), rng.uniform(0.5, 5.0)
            c = torch.distributions.Beta(torch.tensor(a, device=device), torch.tensor(b, device=device)).sample((N,))
            c = c * 4 - 2
        else:
            df = rng.uniform(3, 8)
            z = torch.randn(N, generator=gen, device=device)
            chi = torch.distributions.Chi2(torch.tensor(df, device=device)).sample((N,))
            c = z / torch.sqrt(chi / df)
        cols.append(c)
    return torch.stack(cols, -1) if cols else torch.zeros(N, 0, device=device)


def _categorical(N, card, rng, gen, device, zipf=False):
    """Integer codes 0..card-1 (uniform-ish or Zipf-like frequencies)."""
    if zipf:
        a = rng.uniform(1.1, 2.0)
        p = torch.tensor(np.arange(1, card + 1, dtype=np.float64) ** (-a), device=device, dtype=torch.float32)
    else:
        p = torch.rand(card, generator=gen, device=device) + 0.05
    return torch.multinomial(p / p.sum(), N, replacement=True, generator=gen).float()


def _correlate(X, rho, gen):
    """Mix the columns of X towards a shared factor (pairwise correlation ~rho)."""
    if X.shape[1] < 2:
        return X
    z = torch.randn(X.shape[0], 1, generator=gen, device=X.device)
    return math.sqrt(max(1 - rho, 0.0)) * X + math.sqrt(rho) * z


def calibrate_r2(signal, noise, r2, fit_rows):
    """signal + s * noise with s chosen so the context rows' R^2 of the signal is ``r2``."""
    if r2 >= 1.0:
        return signal
    sig = signal - signal[:fit_rows].mean()
    nz = torch.nan_to_num(noise) - torch.nan_to_num(noise)[:fit_rows].mean()
    ss = float((sig[:fit_rows] ** 2).sum())
    nn_ = float((nz[:fit_rows] ** 2).sum())
    if ss <= 1e-12 or nn_ <= 1e-12:
        return signal
    s = math.sqrt(ss * (1.0 - r2) / (r2 * nn_))
    return signal + s * nz


def _random_fn(v, rng):
    """A random smooth / saturating / periodic univariate function."""
    k = int(rng.integers(0, 7))
    a = rng.uniform(0.5, 2.0)
    if k == 0:
        return torch.tanh(a * v)
    if k == 1:
        return torch.sin(a * v + rng.uniform(0, 6.28))
    if k == 2:
        return v * v * rng.choice([-1.0, 1.0]) * 0.5
    if k == 3:
        return torch.exp(-(a * v) ** 2)
    if k == 4:
        return torch.relu(v - rng.normal(0, 0.5))
    if k == 5:
        return torch.log1p(torch.abs(a * v)) * torch.sign(v)
    return v


# ------------------------------------------------------------------ families
def fam_tree(N, F, fit_rows, rng, gen, device):
    n_cat = int(F * rng.uniform(0.2, 0.6))
    X = torch.cat([_continuous(N, F - n_cat, rng, gen, device),
                   torch.stack([_categorical(N, int(rng.integers(2, 20)), rng, gen, device) for _ in range(n_cat)], -1)
                   if n_cat else torch.zeros(N, 0, device=device)], -1)
    n_trees = int(rng.integers(3, 11))
    y = torch.zeros(N, device=device)
    ctx = X[:fit_rows]
    for _ in range(n_trees):
        depth = int(rng.integers(2, 6))
        node = torch.zeros(N, dtype=torch.long, device=device)
        for level in range(depth):
            n = 2 ** level
            f = torch.tensor(rng.integers(0, F, n), device=device)
            q = torch.rand(n, generator=gen, device=device).clamp(0.05, 0.95)
            thr = torch.quantile(ctx[:, f], q, dim=0).diagonal()
            node = 2 * node + (X.gather(1, f[node].view(-1, 1)).squeeze(1) > thr[node]).long()
        y = y + torch.randn(2 ** depth, generator=gen, device=device)[node]
    y = y / n_trees
    return X, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.6, 0.98), fit_rows)


def fam_gp(N, F, fit_rows, rng, gen, device):
    X = _standardize_cols(_continuous(N, F, rng, gen, device), fit_rows)
    n_act = int(rng.integers(min(2, F), min(max(2, min(8, fit_rows // 32)), F) + 1))
    act = torch.tensor(rng.choice(F, n_act, replace=False), device=device)
    if rng.random() < 0.8 and n_act >= 3:
        X[:, act] = _correlate(X[:, act], rng.uniform(0.15, 0.5), gen)
    Xa = X[:, act]
    M = 512
    ls = torch.tensor(np.exp(rng.uniform(np.log(0.3), np.log(3.0), n_act)), device=device, dtype=torch.float32)
    kind = rng.choice(["rbf", "matern32", "matern52"])
    w = torch.randn(M, n_act, generator=gen, device=device)
    if kind != "rbf":  # Student-t spectral density
        df = 3.0 if kind == "matern32" else 5.0
        chi = torch.distributions.Chi2(torch.tensor(df, device=device)).sample((M, 1))
        w = w / torch.sqrt(chi / df)
    w = w / ls
    b = torch.rand(M, generator=gen, device=device) * 2 * math.pi
    a = torch.randn(M, generator=gen, device=device) * math.sqrt(2.0 / M)
    y = torch.cos(Xa @ w.T + b) @ a
    return X, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.7, 0.99), fit_rows)


def fam_quadratic(N, F, fit_rows, rng, gen, device):
    X = _standardize_cols(_continuous(N, F, rng, gen, device), fit_rows)
    cap = max(1, int((math.sqrt(1 + 8 * max(1, fit_rows // 5)) - 1) / 2))
    n_act = int(rng.integers(min(2, F), max(min(20, F, cap), min(2, F)) + 1))
    act = torch.tensor(rng.choice(F, n_act, replace=False), device=device)
    Xa = X[:, act]
    A = rng.standard_normal((n_act, n_act))
    ev, evec = np.linalg.eigh((A + A.T) / 2)
    ev = ev / max(np.abs(ev).max(), 1e-8) * rng.uniform(0.3, 1.0, n_act)
    Mq = torch.tensor((evec * ev) @ evec.T, device=device, dtype=torch.float32)
    wl = torch.tensor(rng.standard_normal(n_act) * 0.5, device=device, dtype=torch.float32)
    y = ((Xa @ Mq) * Xa).sum(1) + Xa @ wl + rng.standard_normal() * 0.1
    if rng.random() < 0.3 and n_act >= 3:
        for j in rng.choice(n_act, int(rng.integers(1, min(4, n_act))), replace=False):
            y = y + rng.standard_normal() * 0.2 * Xa[:, j] ** 3
    return X, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.7, 0.99), fit_rows)


def fam_sparse_nonlinear(N, F, fit_rows, rng, gen, device):
    n_blocks = int(rng.integers(1, max(2, F // 5) + 1))
    block = torch.tensor(rng.integers(0, n_blocks, F), device=device)
    z = torch.randn(N, n_blocks, generator=gen, device=device)
    rho = torch.tensor(rng.uniform(0.3, 0.95, F), device=device, dtype=torch.float32)
    X = rho * z[:, block] + torch.sqrt(1 - rho * rho) * torch.randn(N, F, generator=gen, device=device)
    for j in np.flatnonzero(rng.random(F) < 0.15):  # descriptor-like transforms
        t = int(rng.integers(0, 4))
        c = X[:, j]
        X[:, j] = c * c if t == 0 else (torch.log1p(c.abs()) if t == 1 else
                                         (torch.round(c * 2) / 2 if t == 2 else torch.tanh(c)))
    n_strong = int(rng.integers(1, min(6, F) + 1))
    strong = rng.choice(F, n_strong, replace=False)
    y = torch.zeros(N, device=device)
    for j in strong:
        y = y + rng.uniform(0.5, 2.0) * _random_fn(X[:, j], rng)
    if n_strong >= 2 and rng.random() < 0.5:
        i, k = rng.choice(strong, 2, replace=False)
        y = y + rng.normal(0, 0.7) * X[:, i] * X[:, k]
    weak = rng.choice(F, min(F, int(rng.integers(0, 10)) + 1), replace=False)
    y = y + X[:, weak] @ torch.tensor(rng.normal(0, 0.1, len(weak)), device=device, dtype=torch.float32)
    if rng.random() < 0.3:  # threshold regime
        j = int(rng.choice(strong))
        y = y + rng.normal(0, 1.0) * (X[:, j] > float(X[:fit_rows, j].median())).float()
    noise = torch.randn(N, generator=gen, device=device)
    if rng.random() < 0.5:  # heteroskedastic
        noise = noise * (0.5 + X[:, int(rng.integers(0, F))].abs())
    return X, calibrate_r2(y, noise, rng.uniform(0.5, 0.95), fit_rows)


def fam_lookup(N, F, fit_rows, rng, gen, device):
    n_id = min(int(rng.integers(1, 4)), max(1, F - 1))
    ids, y = [], torch.zeros(N, device=device)
    for _ in range(n_id):
        card = int(rng.integers(10, max(11, min(500, fit_rows // 2))))
        c = _categorical(N, card, rng, gen, device, zipf=True)
        ids.append(c)
        y = y + rng.uniform(0.5, 2.0) * torch.randn(card, generator=gen, device=device)[c.long()]
    n_cont = F - n_id
    Xc = _standardize_cols(_continuous(N, n_cont, rng, gen, device), fit_rows)
    if n_cont:
        w = torch.tensor(rng.normal(0, 0.3, n_cont), device=device, dtype=torch.float32)
        y = y + Xc @ w
    X = torch.cat([torch.stack(ids, -1), Xc], -1)
    return X, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.5, 0.95), fit_rows)


def fam_cat_dominant(N, F, fit_rows, rng, gen, device):
    n_cat = max(min(F, 4), int(round(F * rng.uniform(0.6, 0.95))))
    n_cat = min(n_cat, F)
    cards = [int(min(50, max(2, round(rng.pareto(1.2) * 3 + 2)))) for _ in range(n_cat)]
    C = torch.stack([_categorical(N, k, rng, gen, device) for k in cards], -1)
    imp = rng.dirichlet(np.ones(n_cat) * 0.5)
    y = torch.zeros(N, device=device)
    for j, k in enumerate(cards):
        if rng.random() < 0.5:  # nominal: random per-level effect
            eff = torch.randn(k, generator=gen, device=device)
        else:  # ordinal: monotone effect
            eff = torch.sort(torch.randn(k, generator=gen, device=device)).values * rng.choice([-1.0, 1.0])
        y = y + math.sqrt(imp[j]) * 2 * eff[C[:, j].long()]
    for _ in range(int(rng.integers(0, 5))):
        if n_cat < 2:
            break
        i, j = rng.choice(n_cat, 2, replace=False)
        tab = torch.randn(cards[i], cards[j], generator=gen, device=device) * 0.5
        y = y + tab[C[:, i].long(), C[:, j].long()]
    Xc = _standardize_cols(_continuous(N, F - n_cat, rng, gen, device), fit_rows)
    if F - n_cat:
        y = y + 0.3 * Xc @ torch.tensor(rng.normal(0, 1, F - n_cat), device=device, dtype=torch.float32)
    return torch.cat([C, Xc], -1), calibrate_r2(y, torch.randn(N, generator=gen, device=device),
                                                 rng.uniform(0.45, 0.92), fit_rows)


def fam_binary(N, F, fit_rows, rng, gen, device):
    on = torch.tensor(np.clip(rng.beta(0.5, 4.0, F), 1.0 / max(N, 1), 0.5), device=device, dtype=torch.float32)
    X = (torch.rand(N, F, generator=gen, device=device) < on).float()
    dead = X[:fit_rows].std(0, unbiased=False) < 1e-8
    if bool(dead.any()):  # repair columns with no variation in the context
        X[: max(1, fit_rows // 100), dead] = 1.0 - X[: max(1, fit_rows // 100), dead]
    n_act = int(rng.integers(min(5, F), min(30, F) + 1))
    act = torch.tensor(rng.choice(F, n_act, replace=False), device=device)
    w = torch.tensor(rng.pareto(1.5, n_act) * rng.choice([-1, 1], n_act), device=device, dtype=torch.float32)
    y = X[:, act] @ w
    if rng.random() < 0.4 and n_act >= 2:
        y = y + torch.tanh(X[:, act[:2]].sum(1) - 1.0) * rng.normal(0, 1.0)
    return X, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.4, 0.9), fit_rows)


def fam_temporal(N, F, fit_rows, rng, gen, device):
    t = torch.linspace(0, 1, N, device=device)
    mode = int(rng.integers(0, 5))
    eps = torch.randn(N, F, generator=gen, device=device)
    rho = torch.tensor(rng.uniform(0.5, 0.99, F), device=device, dtype=torch.float32)
    # AR(1) features by a scan in log2(N) doubling steps: x_t = rho x_{t-1} + e_t
    X = eps.clone()
    step, coef = 1, rho.clone()
    while step < N:
        X[step:] = X[step:] + coef * X[:-step]
        coef = coef * coef
        step *= 2
    X = X * torch.sqrt(1 - rho * rho)
    w = torch.tensor(rng.normal(0, 1, F), device=device, dtype=torch.float32) * (
        torch.tensor(rng.random(F) < min(1.0, 6.0 / F), device=device).float())
    if mode == 1:  # lagged features drive y
        lag = int(rng.integers(1, 6))
        Xl = torch.cat([X[:1].expand(lag, F), X[:-lag]], 0)
        y = Xl @ w
    elif mode == 2:  # concept drift
        w2 = w + torch.tensor(rng.normal(0, 1, F), device=device, dtype=torch.float32) * (w != 0).float()
        y = ((1 - t).unsqueeze(1) * X * w + t.unsqueeze(1) * X * w2).sum(1)
    elif mode == 3:  # trend + seasonal features
        per = rng.uniform(0.05, 0.5)
        X[:, 0] = torch.sin(2 * math.pi * t / per)
        if F > 1:
            X[:, 1] = torch.cos(2 * math.pi * t / per)
        y = X @ w + rng.normal(0, 1.0) * X[:, 0] + rng.normal(0, 2.0) * t
    elif mode == 4:  # pure trend on y
        y = rng.normal(0, 3.0) * t + X @ w
    else:
        y = X @ w + 0.5 * torch.tanh(X @ w)
    return _standardize_cols(X, fit_rows), calibrate_r2(y, torch.randn(N, generator=gen, device=device),
                                                        rng.uniform(0.5, 0.95), fit_rows)


def fam_clean_lowdim(N, F, fit_rows, rng, gen, device):
    Fa = min(F, int(rng.integers(5, 31)))
    n_cat = int(round(Fa * rng.uniform(0.3, 0.8)))
    C = [_categorical(N, int(rng.integers(2, 12)), rng, gen, device) for _ in range(n_cat)]
    Xc = _standardize_cols(_continuous(N, Fa - n_cat, rng, gen, device), fit_rows)
    X = torch.cat([torch.stack(C, -1) if C else torch.zeros(N, 0, device=device), Xc], -1)
    y = torch.zeros(N, device=device)
    for _ in range(int(rng.integers(1, 4))):  # a few simple rules
        j = int(rng.integers(0, Fa))
        thr = float(X[:fit_rows, j].median())
        y = y + rng.normal(0, 1.5) * (X[:, j] > thr).float()
    if Fa - n_cat:
        y = y + Xc @ torch.tensor(rng.normal(0, 0.5, Fa - n_cat), device=device, dtype=torch.float32)
    out = torch.zeros(N, F, device=device)
    out[:, :Fa] = X
    return out, calibrate_r2(y, torch.randn(N, generator=gen, device=device), rng.uniform(0.85, 0.99), fit_rows)


FAMILIES = {"tree": fam_tree, "gp": fam_gp, "quadratic": fam_quadratic, "sparse_nonlinear": fam_sparse_nonlinear,
            "lookup": fam_lookup, "cat_dominant": fam_cat_dominant, "binary": fam_binary, "temporal": fam_temporal,
            "clean_lowdim": fam_clean_lowdim}


# ------------------------------------------------------------------ augmentations
def augment_table(X, F, fit_rows, rng, gen, p_episode=0.6, p_col=0.4, missing_prob=0.5, heavy_prob=0.3,
                  cat_prob=0.2):
    """In-place feature augmentation of one table ``X [N, F_pad]`` (first F columns live)."""
    N = X.shape[0]
    dev = X.device
    if rng.random() < p_episode:  # per-column monotone shape transforms, then re-standardise
        for j in range(F):
            if rng.random() >= p_col:
                continue
            c = X[:, j]
            if torch.unique(c[:fit_rows]).numel() < min(20, max(2, N // 50)):
                continue  # keep categorical-looking columns as they are
            k = int(rng.integers(0, 6))
            if k == 0:
                c = torch.expm1(c.clamp(-10, 10) * rng.uniform(0.3, 1.0))
            elif k == 1:
                c = torch.sign(c) * torch.log1p(c.abs() * rng.uniform(0.5, 3.0))
            elif k == 2:
                c = torch.sign(c) * c.abs() ** rng.uniform(1.5, 3.0)
            elif k == 3:
                c = torch.argsort(torch.argsort(c)).float() / max(N - 1, 1)
            elif k == 4:
                c = -c
            else:
                c = c * c
            ref = c[:fit_rows]
            sd = ref.std(unbiased=False)
            X[:, j] = (c - ref.mean()) / sd if float(sd) > 1e-8 else c - ref.mean()
    if rng.random() < cat_prob and F > 1:  # numeric -> categorical codes (random level order)
        for j in rng.choice(F, max(1, int(F * rng.uniform(0.05, 0.3))), replace=False):
            k = int(rng.integers(2, 20))
            q = torch.quantile(X[:fit_rows, j], torch.linspace(0, 1, k + 1, device=dev)[1:-1])
            codes = torch.bucketize(X[:, j].contiguous(), q)
            perm = torch.randperm(k, generator=gen, device=dev)
            X[:, j] = perm[codes].float()
    if rng.random() < heavy_prob:  # heavy-tailed spikes in a few columns
        for j in rng.choice(F, max(1, int(F * rng.uniform(0.1, 0.5))), replace=False):
            m = torch.rand(N, generator=gen, device=dev) < rng.uniform(0.005, 0.05)
            df = rng.uniform(1.5, 4.0)
            chi = torch.distributions.Chi2(torch.tensor(df, device=dev)).sample((N,))
            spikes = torch.randn(N, generator=gen, device=dev) / torch.sqrt(chi / df) * rng.uniform(3, 10)
            X[:, j] = torch.where(m, X[:, j] + spikes, X[:, j])
    if rng.random() < missing_prob:
        if rng.random() < 0.5:  # missing completely at random
            rate = rng.uniform(0.01, 0.3)
            cols = torch.tensor(rng.random(F) < rng.uniform(0.2, 1.0), device=dev)
            m = (torch.rand(N, F, generator=gen, device=dev) < rate) & cols
            X[:, :F] = torch.where(m, torch.full_like(X[:, :F], float("nan")), X[:, :F])
        elif F > 1:  # missing where another column is in its context tail
            drv = int(rng.integers(0, F))
            tgt = [c for c in rng.choice(F, min(3, F), replace=False) if c != drv]
            p = rng.uniform(75, 95)
            thr = torch.quantile(X[:fit_rows, drv], p / 100.0)
            m = X[:, drv] > thr if rng.random() < 0.5 else X[:, drv] < torch.quantile(X[:fit_rows, drv], 1 - p / 100)
            for c in tgt:
                X[:, c] = torch.where(m & (torch.rand(N, generator=gen, device=dev) < 0.8),
                                      torch.full_like(X[:, c], float("nan")), X[:, c])
    return X


# ------------------------------------------------------------------ batch
def generate_batch(batch_size: int, n_rows: int, eval_pos: int, seed: int, device, min_features: int = 5,
                   max_features: int = 100, pad_features: int = 100, family_probs: dict | None = None,
                   augment: bool = True):
    """``(X [B, N, pad] with NaN for missing cells, y [B, N] standardised on the context,
    n_features [B], families)`` from the prior mixture."""
    from synthefy_nori_b200.training.scm_prior import scm_prior_tables

    rng = np.random.default_rng(int(seed))
    gen = torch.Generator(device=device).manual_seed(int(rng.integers(0, 2 ** 62)))
    probs = dict(family_probs or DEFAULT_FAMILY_PROBS)
    names = list(probs)
    p = np.array([probs[k] for k in names], dtype=np.float64)
    p = p / p.sum()
    fam = [names[i] for i in rng.choice(len(names), batch_size, p=p)]
    n_feat = [int(rng.integers(min_features, max_features + 1)) for _ in range(batch_size)]
    X = torch.zeros(batch_size, n_rows, pad_features, device=device)
    y = torch.zeros(batch_size, n_rows, device=device)
    scm_idx = [i for i, f in enumerate(fam) if f == "scm"]
    if scm_idx:
        xs, ys, _ = scm_prior_tables(len(scm_idx), n_rows, [n_feat[i] for i in scm_idx], eval_pos,
                                     int(rng.integers(0, 2 ** 62)), device, pad_features=pad_features)
        X[scm_idx] = xs
        y[scm_idx] = ys
    for i, f in enumerate(fam):
        if f == "scm":
            continue
        xf, yf = FAMILIES[f](n_rows, n_feat[i], eval_pos, rng, gen, device)
        X[i, :, : xf.shape[1]] = xf
        y[i] = yf
    if augment:  # True, or a dict of augment_table probabilities
        kw = augment if isinstance(augment, dict) else {}
        for i in range(batch_size):
            augment_table(X[i], n_feat[i], eval_pos, rng, gen, **kw)
    y = torch.nan_to_num(y)
    mu = y[:, :eval_pos].mean(1, keepdim=True)
    sd = y[:, :eval_pos].std(1, unbiased=False, keepdim=True)
    y = torch.where(sd > 1e-8, (y - mu) / sd.clamp(min=1e-8), y - mu).clamp(-1e4, 1e4)
    X[:, :, :] = torch.where(torch.isinf(X), torch.full_like(X, float("nan")), X)
    return X, y, torch.tensor(n_feat, device=device), fam
