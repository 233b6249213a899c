"""Batched SCM prior on the GPU: many random structural causal models per launch.

Behaviour follows the reference prior (``training/scm_prior_generator.py``): every table
draws its own hyperparameters from meta-distributions (MLP vs tree SCM, causal or not,
number of causes, depth, width, weight scale, noise, root sampling, block-wise dropout,
activation); an MLP SCM propagates sampled root causes through random layers
``act(scale * (standardise(h) + shift)) W^T + b + noise`` clamped to +-100; features and
the target are picked among the hidden units (causal) or are the roots and the output
(non-causal); a tree SCM passes the roots through 1-2 layers of random shallow trees.
Features are then stabilised with context-row median / MAD, constant columns zeroed,
and the target standardised with context statistics.

B200 design: the hyperparameters are drawn on the host (a few dozen numbers per table),
everything else is batched over the tables of a step on the device.  Tables are padded
to a common width; the activation and the noisy linear map of every layer run as one
``scm_act`` + one ``scm_linear`` launch for the whole batch (``csrc/prior.cu``: fp32
tiled GEMM, counter-based Gaussian noise, fp64 context-row column sums for the next
layer's standardisation), instead of a Python loop of small per-table modules.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

ACTIVATIONS = ("tanh", "leaky_relu", "elu", "identity", "selu", "silu", "relu", "softplus", "relu6", "hardtanh",
               "sign", "rbf", "exp", "sqrt_abs", "unit_interval", "sin", "square", "abs", "random_fourier")
RFF = ACTIVATIONS.index("random_fourier")
N_SIMPLE = 18
# the reference's factory list: 18 simple activations + 10 copies of the random-Fourier
# one (each wrapped in standardise -> random affine), then as many "pick one of those
# per layer" entries
N_FIXED = N_SIMPLE + 10
N_FACTORIES = 2 * N_FIXED
MAX_HIDDEN = 512  # width cap of the padded batch (the meta-distribution's far tail is clipped here)


def _factory_act(f: int) -> int | None:
    """Activation code of a fixed factory, None for a per-layer random-choice factory."""
    if f < N_SIMPLE:
        return f
    if f < N_FIXED:
        return RFF
    return None


# ------------------------------------------------------------------ meta-distributions
def _trunc_norm_log_scaled(rng, min_mean, max_mean, lower_bound=0.0, round_val=False):
    mu = math.exp(rng.uniform(math.log(max(min_mean, 1e-8)), math.log(max(max_mean, 1e-7))))
    sigma = mu * math.exp(rng.uniform(math.log(0.01), math.log(1.0)))
    if round_val:
        v = max(rng.normal(mu, max(sigma, 1e-8)), lower_bound)
        return max(int(round(v)), int(math.ceil(lower_bound)))
    for _ in range(64):  # a truly truncated draw (no atom at the bound)
        v = rng.normal(mu, max(sigma, 1e-8))
        if v > lower_bound:
            return float(v)
    return max(mu, float(np.nextafter(lower_bound, math.inf)))


def _meta_choice(rng, values):
    w = np.concatenate([[1.0], rng.uniform(-3, 5, len(values) - 1)])
    p = np.exp(w - w.max())
    return values[rng.choice(len(values), p=p / p.sum())]


def _meta_beta(rng, scale=1.0, min_b=0.1, max_b=5.0, min_k=0.1, max_k=5.0):
    return float(rng.beta(rng.uniform(min_b, max_b), rng.uniform(min_k, max_k)) * scale)


def _activation_factory(rng) -> int:
    w = np.concatenate([[1.0], rng.uniform(-5, 6, N_FACTORIES - 1)])
    p = np.exp(w - w.max())
    return int(rng.choice(N_FACTORIES, p=p / p.sum()))


@dataclass
class SCMHyper:
    scm_type: str
    is_causal: bool
    num_causes: int
    y_is_effect: bool
    in_clique: bool
    sort_features: bool
    num_layers: int
    hidden_dim: int
    init_std: float
    noise_std: float
    sampling: str
    pre_sample_cause_stats: bool
    pre_sample_noise_std: bool
    block_wise_dropout: bool
    dropout_prob: float
    act_factory: int


def sample_hyperparams(rng: np.random.Generator, mlp_prob: float = 0.7) -> SCMHyper:
    """One table's SCM hyperparameters from the meta-distributions."""
    return SCMHyper(
        scm_type="mlp" if rng.random() < mlp_prob else "tree",
        is_causal=bool(_meta_choice(rng, [True, False])),
        num_causes=int(_trunc_norm_log_scaled(rng, 1, 12, lower_bound=1, round_val=True)),
        y_is_effect=bool(_meta_choice(rng, [True, False])),
        in_clique=bool(_meta_choice(rng, [True, False])),
        sort_features=bool(_meta_choice(rng, [True, False])),
        num_layers=int(_trunc_norm_log_scaled(rng, 1, 6, lower_bound=2, round_val=True)),
        hidden_dim=int(_trunc_norm_log_scaled(rng, 5, 130, lower_bound=4, round_val=True)),
        init_std=_trunc_norm_log_scaled(rng, 0.01, 10.0),
        noise_std=_trunc_norm_log_scaled(rng, 0.0001, 0.3),
        sampling=str(_meta_choice(rng, ["normal", "mixed", "uniform"])),
        pre_sample_cause_stats=bool(_meta_choice(rng, [True, False])),
        pre_sample_noise_std=bool(_meta_choice(rng, [True, False])),
        block_wise_dropout=bool(_meta_choice(rng, [True, False])),
        dropout_prob=_meta_beta(rng, scale=0.9),
        act_factory=_activation_factory(rng),
    )


# ------------------------------------------------------------------ roots
def _zipf_table(a: float, kmax: int = 10, terms: int = 4000) -> np.ndarray:
    """P(min(Zipf(a), kmax) = k) for k = 1..kmax (zeta normaliser summed + integral tail)."""
    k = np.arange(1, terms + 1, dtype=np.float64)
    w = k ** (-a)
    zeta = w.sum() + terms ** (1 - a) / (a - 1)
    p = w[: kmax - 1] / zeta
    return np.concatenate([p, [max(1.0 - p.sum(), 0.0)]])


def sample_roots(rng: np.random.Generator, hp: SCMHyper, n_cols: int, N: int, fit_rows: int, gen: torch.Generator,
                 device) -> torch.Tensor:
    """Root causes ``[N, n_cols]`` (normal / uniform / mixed per column)."""
    if hp.sampling == "uniform":
        return torch.rand(N, n_cols, generator=gen, device=device)
    if hp.sampling == "normal" or n_cols == 0:
        z = torch.randn(N, n_cols, generator=gen, device=device)
        if hp.pre_sample_cause_stats:
            means = rng.normal(0, 1, n_cols)
            stds = np.abs(rng.normal(0, 1, n_cols) * means)
            z = z * torch.tensor(stds, device=device, dtype=torch.float32) + torch.tensor(means, device=device,
                                                                                         dtype=torch.float32)
        return z
    # mixed: per column normal, multinomial, Zipf or uniform
    zipf_p, multi_p, normal_p = rng.random() * 0.66, rng.random() * 0.66, rng.random() * 0.66
    cols = []
    for _ in range(n_cols):
        if rng.random() > normal_p:
            cols.append(torch.randn(N, generator=gen, device=device))
        elif rng.random() > multi_p:
            probs = torch.rand(int(rng.integers(2, 20)), generator=gen, device=device)
            x = torch.multinomial(probs, N, replacement=True, generator=gen).float()
            ref = x[:fit_rows]
            sd = ref.std() if fit_rows > 1 else torch.zeros((), device=device)
            cols.append((x - ref.mean()) / sd.clamp(min=1e-6))
        elif rng.random() > zipf_p:
            p = _zipf_table(2.0 + rng.random() * 2.0)
            x = torch.multinomial(torch.tensor(p, device=device, dtype=torch.float32), N, replacement=True,
                                  generator=gen).float() + 1.0
            cols.append(x - x[:fit_rows].mean())
        else:
            cols.append(torch.rand(N, generator=gen, device=device))
    return torch.stack(cols, -1)


# ------------------------------------------------------------------ weights
def block_dropout_weight(rng, out_dim: int, in_dim: int, init_std: float, dropout_prob: float,
                         gen: torch.Generator, device) -> torch.Tensor:
    """``[out_dim, in_dim]``: balanced diagonal blocks, element dropout inside them with at
    least one kept connection per row and column, std scaled by 1 / sqrt(keep fraction)."""
    n_blocks = int(rng.integers(1, math.ceil(math.sqrt(min(out_dim, in_dim))) + 1))

    def block_ids(size):
        q, r = divmod(size, n_blocks)
        widths = [q + (1 if i < r else 0) for i in range(n_blocks)]
        return torch.repeat_interleave(torch.arange(n_blocks, device=device), torch.tensor(widths, device=device)), widths

    rb, rw = block_ids(out_dim)
    cb, cw = block_ids(in_dim)
    inblock = rb.view(-1, 1) == cb.view(1, -1)
    keep = (torch.rand(out_dim, in_dim, generator=gen, device=device) >= dropout_prob) & inblock
    cstart = torch.tensor(np.concatenate([[0], np.cumsum(cw)[:-1]]), device=device)
    rstart = torch.tensor(np.concatenate([[0], np.cumsum(rw)[:-1]]), device=device)
    cwt, rwt = torch.tensor(cw, device=device), torch.tensor(rw, device=device)
    dead_r = ~keep.any(1)
    if bool(dead_r.any()):
        j = cstart[rb] + (torch.rand(out_dim, generator=gen, device=device) * cwt[rb]).long().clamp(max=cwt[rb] - 1)
        keep[torch.arange(out_dim, device=device)[dead_r], j[dead_r]] = True
    dead_c = ~keep.any(0)
    if bool(dead_c.any()):
        i = rstart[cb] + (torch.rand(in_dim, generator=gen, device=device) * rwt[cb]).long().clamp(max=rwt[cb] - 1)
        keep[i[dead_c], torch.arange(in_dim, device=device)[dead_c]] = True
    frac = float(keep.sum()) / float(out_dim * in_dim)
    std = init_std / math.sqrt(max(frac, 1e-12))
    return torch.randn(out_dim, in_dim, generator=gen, device=device) * std * keep


def _weight(rng, hp, out_dim, in_dim, gen, device):
    if hp.block_wise_dropout:
        return block_dropout_weight(rng, out_dim, in_dim, hp.init_std, hp.dropout_prob, gen, device)
    return torch.randn(out_dim, in_dim, generator=gen, device=device) * hp.init_std


# ------------------------------------------------------------------ MLP SCM (batched)
_TORCH_ACTS = (torch.tanh, lambda x: torch.nn.functional.leaky_relu(x, 0.01), torch.nn.functional.elu, lambda x: x,
               torch.nn.functional.selu, torch.nn.functional.silu, torch.relu, torch.nn.functional.softplus,
               torch.nn.functional.relu6, torch.nn.functional.hardtanh, lambda x: 2 * (x >= 0).float() - 1,
               lambda x: torch.exp(-x * x), torch.exp, lambda x: torch.sqrt(x.abs()), lambda x: (x.abs() <= 1).float(),
               torch.sin, lambda x: x * x, torch.abs)


class _TorchKernels:
    """Plain-tensor statement of ``scm_act`` / ``scm_linear`` (CPU generation, e.g. in
    prefetch worker processes).  The noise comes from a torch generator instead of the
    kernel's counter hash, so values differ from the device path draw for draw."""

    @staticmethod
    def scm_act(h, code, scale, shift, width, mean, rstd, rff):
        B, N, H = h.shape
        z = (h - mean.unsqueeze(1)) * rstd.unsqueeze(1)
        out = torch.zeros_like(h)
        for b in range(B):
            w = int(width[b])
            c = int(code[b])
            if w == 0:
                continue
            if c == RFF:
                v = (rff[b, 2] * torch.sin(rff[b, 0] * z[b, :, :w].unsqueeze(-1) + rff[b, 1])).sum(-1)
            else:
                v = _TORCH_ACTS[c](scale[b] * (z[b, :, :w] + shift[b]))
            out[b, :, :w] = torch.where(torch.isfinite(v), v, torch.zeros_like(v))
        return out

    @staticmethod
    def scm_linear(A, W, bias, sigma, out_width, fit_rows, seed, layer, csum, csq):
        g = torch.Generator(device=A.device).manual_seed((int(seed) + 7919 * layer) & 0x7FFFFFFFFFFFFFFF)
        h = torch.bmm(A, W.transpose(1, 2)) + bias.unsqueeze(1)
        h = h + sigma.unsqueeze(1) * torch.randn(h.shape, generator=g, device=A.device)
        h = torch.where(torch.isfinite(h), h.clamp(-100, 100), torch.zeros_like(h))
        cols = torch.arange(h.shape[-1], device=A.device).view(1, 1, -1)
        h = h * (cols < out_width.view(-1, 1, 1)).float()
        csum += h[:, :fit_rows].double().sum(1)
        csq += (h[:, :fit_rows].double() ** 2).sum(1)
        return h


def mlp_scm_batch(hps: list[SCMHyper], n_features: list[int], N: int, fit_rows: int, seed: int, device,
                  rng: np.random.Generator):
    """Raw (X [B, N, Fmax], y [B, N]) of a batch of MLP SCMs (native kernels on CUDA)."""
    if torch.device(device).type == "cuda":
        from synthefy_nori_b200 import ops

        C = ops.lib()
    else:
        C = _TorchKernels
    B = len(hps)
    gen = torch.Generator(device=device).manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    causes, hidden, depth = [], [], []
    for hp, F in zip(hps, n_features):
        causes.append(hp.num_causes if hp.is_causal else F)
        h = max(hp.hidden_dim, 1 + 2 * F) if hp.is_causal else hp.hidden_dim
        hidden.append(min(h, MAX_HIDDEN))
        depth.append(hp.num_layers)
    Cmax = -(-max(causes) // 4) * 4
    Hmax = -(-max(hidden) // 32) * 32
    # per-layer widths: layer 0 = Linear(causes -> hidden); 1..L-1 hidden -> hidden; the
    # non-causal output layer (L) hidden -> 1
    n_lin = max(d + (0 if hp.is_causal else 1) for d, hp in zip(depth, hps))
    roots = torch.zeros(B, N, Cmax, device=device)
    for b, hp in enumerate(hps):
        roots[b, :, : causes[b]] = sample_roots(rng, hp, causes[b], N, fit_rows, gen, device)
    # per-layer activation codes (a random-choice factory draws one per layer)
    codes = np.zeros((n_lin, B), np.int32)
    scales = np.ones((n_lin, B), np.float32)
    shifts = np.zeros((n_lin, B), np.float32)
    for b, hp in enumerate(hps):
        fixed = _factory_act(hp.act_factory)
        for layer in range(n_lin):
            f = fixed if fixed is not None else _factory_act(int(rng.integers(0, N_FIXED)))
            codes[layer, b] = f
            scales[layer, b] = math.exp(2.0 * rng.standard_normal())
            shifts[layer, b] = rng.standard_normal()
    outs = []
    h = None
    csum = csq = None
    for layer in range(n_lin):
        in_dim = Cmax if layer == 0 else Hmax
        W = torch.zeros(B, Hmax, in_dim, device=device)
        sigma = torch.zeros(B, Hmax, device=device)
        width = np.zeros(B, np.int32)
        for b, hp in enumerate(hps):
            last = depth[b] + (0 if hp.is_causal else 1)
            if layer >= last:
                continue
            out_w = 1 if (not hp.is_causal and layer == depth[b]) else hidden[b]
            k_in = causes[b] if layer == 0 else hidden[b]
            W[b, :out_w, :k_in] = _weight(rng, hp, out_w, k_in, gen, device)
            if layer > 0 and hp.noise_std > 0:
                if hp.pre_sample_noise_std:
                    ns = np.maximum(np.abs(rng.normal(0.0, hp.noise_std, out_w)), np.finfo(np.float32).eps)
                    sigma[b, :out_w] = torch.tensor(ns, device=device, dtype=torch.float32)
                else:
                    sigma[b, :out_w] = hp.noise_std
            width[b] = out_w
        width_t = torch.tensor(width, device=device)
        if layer == 0:
            A = roots
        else:
            n = max(fit_rows, 1)
            mean = (csum / n).float()
            var = ((csq - csum * csum / n) / max(n - 1, 1)).clamp(min=0) if fit_rows > 1 else torch.zeros_like(csum)
            rstd = (1.0 / (var.sqrt() + 1e-6)).float()
            rff = torch.zeros(B, 3, 256, device=device)
            for b in range(B):
                if codes[layer, b] == RFF:
                    fr = 256 * torch.rand(256, generator=gen, device=device)
                    ph = 2 * math.pi * torch.rand(256, generator=gen, device=device)
                    decay = -math.exp(rng.uniform(math.log(0.7), math.log(3.0)))
                    fac = fr.clamp_min(torch.finfo(torch.float32).eps) ** decay
                    fac = fac / (fac * fac).sum().sqrt()
                    rff[b] = torch.stack([fr, ph, fac * torch.randn(256, generator=gen, device=device)])
            in_width = torch.tensor([hidden[b] if layer < depth[b] + (0 if hps[b].is_causal else 1) else 0
                                     for b in range(B)], dtype=torch.int32, device=device)
            A = C.scm_act(h, torch.tensor(codes[layer], device=device), torch.tensor(scales[layer], device=device),
                          torch.tensor(shifts[layer], device=device), in_width, mean.contiguous(), rstd.contiguous(),
                          rff)
        csum = torch.zeros(B, Hmax, device=device, dtype=torch.float64)
        csq = torch.zeros_like(csum)
        h = C.scm_linear(A.contiguous(), W, torch.zeros(B, Hmax, device=device), sigma, width_t, fit_rows,
                         int(rng.integers(0, 2 ** 62)), layer, csum, csq)
        outs.append(h)
    return _select_outputs(hps, n_features, outs, roots, causes, hidden, depth, N, device, rng)


def _select_outputs(hps, n_features, outs, roots, causes, hidden, depth, N, device, rng):
    B = len(hps)
    Fmax = max(n_features)
    stack = torch.stack(outs)  # [L, B, N, H]
    li = np.zeros((B, Fmax), np.int64)
    ci = np.zeros((B, Fmax), np.int64)
    yl, yc = np.zeros(B, np.int64), np.zeros(B, np.int64)
    from_roots = np.zeros(B, bool)
    for b, hp in enumerate(hps):
        F = n_features[b]
        if not hp.is_causal:
            from_roots[b] = True
            yl[b], yc[b] = depth[b], 0  # the output layer
            continue
        hb = hidden[b]
        total = (depth[b] - 1) * hb  # hidden units of layers 1 .. depth-1 (the outputs after the first projection)
        if hp.in_clique:
            start = int(rng.integers(0, max(0, total - 1 - F) + 1))
            perm = start + rng.permutation(1 + F)
        else:
            perm = rng.permutation(max(total - 1, 1))
        ix = perm[1 : 1 + F]
        iy = total - 1 if hp.y_is_effect else perm[0]
        if hp.sort_features:
            ix = np.sort(ix)
        ix = np.clip(ix, 0, total - 1)
        iy = int(np.clip(iy, 0, total - 1))
        li[b, : len(ix)] = 1 + ix // hb
        ci[b, : len(ix)] = ix % hb
        yl[b], yc[b] = 1 + iy // hb, iy % hb
    lt, ct = torch.tensor(li, device=device), torch.tensor(ci, device=device)
    bt = torch.arange(B, device=device).view(B, 1).expand(B, Fmax)
    X = stack[lt, bt, :, ct].permute(0, 2, 1).contiguous()  # [B, N, Fmax]
    y = stack[torch.tensor(yl, device=device), torch.arange(B, device=device), :, torch.tensor(yc, device=device)]
    for b in range(B):
        if from_roots[b]:
            X[b, :, : n_features[b]] = roots[b, :, : n_features[b]]
        X[b, :, n_features[b]:] = 0.0
    return X, y


# ------------------------------------------------------------------ tree SCM (batched tensor program)
def tree_scm_batch(hps: list[SCMHyper], n_features: list[int], N: int, fit_rows: int, seed: int, device,
                   rng: np.random.Generator):
    """Non-causal tree SCMs: X = roots; y = 1-2 layers of random shallow tree ensembles
    (random feature and a threshold at a random context quantile per node, leaf values
    fitted to a random target: the leaf means of N(0, 1) draws on the context rows), plus
    noise.  Per table: layers in {1, 2}, hidden width in [3, 10], depth <= 4, <= 4 trees."""
    B = len(hps)
    gen = torch.Generator(device=device).manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    Fmax = max(n_features)
    X = torch.zeros(B, N, Fmax, device=device)
    y = torch.zeros(B, N, device=device)
    for b, (hp, F) in enumerate(zip(hps, n_features)):
        h = sample_roots(rng, hp, F, N, fit_rows, gen, device)
        X[b, :, :F] = h
        n_layers, width = int(rng.integers(1, 3)), int(rng.integers(3, 11))
        for layer in range(n_layers):
            out_dim = width if layer < n_layers - 1 else 1
            depth_ = min(2 + int(rng.exponential(2.0)), 4)
            n_est = min(1 + int(rng.exponential(2.0)), 4)
            outs = []
            for _ in range(out_dim):
                acc = torch.zeros(N, device=device)
                target = torch.randn(N, generator=gen, device=device)
                for _ in range(n_est):
                    acc = acc + _random_tree(h, depth_, target, fit_rows, gen, rng)
                outs.append(acc)
            h = torch.stack(outs, -1)
            if hp.noise_std > 0:
                h = h + torch.randn(h.shape, generator=gen, device=device) * hp.noise_std
        y[b] = h[:, 0]
    return X, y


def _random_tree(h, depth, target, fit_rows, gen, rng):
    N, D = h.shape
    node = torch.zeros(N, dtype=torch.long, device=h.device)
    ctx = h[:fit_rows]
    for _level in range(depth):
        n_nodes = 2 ** _level
        feat = torch.tensor(rng.integers(0, D, n_nodes), device=h.device)
        q = torch.rand(n_nodes, generator=gen, device=h.device)
        col = ctx[:, feat]  # [fit_rows, n_nodes]
        thr = torch.quantile(col, q.clamp(0.02, 0.98), dim=0).diagonal() if fit_rows > 1 else torch.zeros(n_nodes,
                                                                                                         device=h.device)
        go_right = h.gather(1, feat[node].view(-1, 1)).squeeze(1) > thr[node]
        node = 2 * node + go_right.long()
    leaves = 2 ** depth
    sums = torch.zeros(leaves, device=h.device).index_add_(0, node[:fit_rows], target[:fit_rows])
    cnt = torch.zeros(leaves, device=h.device).index_add_(0, node[:fit_rows], torch.ones(fit_rows, device=h.device))
    val = sums / cnt.clamp(min=1)
    return val[node]


# ------------------------------------------------------------------ post-processing
def stabilize(X: torch.Tensor, y: torch.Tensor, n_features: list[int], fit_rows: int, clip: float = 50.0):
    """Median / MAD feature scaling on the context rows (max-deviation scaling for columns
    whose MAD is ~0, so rare discrete levels stay distinct), constant columns zeroed,
    target standardised with context statistics (clip +-1e4)."""
    X = torch.nan_to_num(X.float(), nan=0.0, posinf=1e6, neginf=-1e6).clamp(-1e6, 1e6)
    ref = X[:, :fit_rows]
    med = ref.median(dim=1, keepdim=True).values
    cen = X - med
    rc = ref - med
    mad = rc.abs().median(dim=1, keepdim=True).values
    bound = rc.abs().amax(dim=1, keepdim=True) / clip
    scale = torch.where(mad < 1e-6, bound, mad).clamp(min=1e-6)
    X = (cen / scale).clamp(-clip, clip)
    if fit_rows > 1:
        const = X[:, :fit_rows].std(dim=1, unbiased=False, keepdim=True) <= 1e-8
        X = torch.where(const, torch.zeros_like(X), X)
    Fpad = X.shape[-1]
    live = torch.arange(Fpad, device=X.device).view(1, 1, -1) < torch.tensor(n_features, device=X.device).view(-1, 1, 1)
    X = torch.where(live, X, torch.zeros_like(X))
    y = torch.nan_to_num(y.float(), nan=0.0, posinf=1e4, neginf=-1e4).clamp(-1e6, 1e6)
    ym = y[:, :fit_rows].mean(1, keepdim=True)
    ys = y[:, :fit_rows].std(1, unbiased=False, keepdim=True)
    y = torch.where(ys > 1e-8, (y - ym) / ys.clamp(min=1e-8), y - ym).clamp(-1e4, 1e4)
    return X, y


def fallback_linear(N: int, F: int, gen: torch.Generator, device):
    """A known-learnable linear table (used when a sampled SCM degenerates)."""
    X = torch.randn(N, F, generator=gen, device=device)
    k = min(F, 4)
    w = torch.arange(k, 0, -1, dtype=torch.float32, device=device)
    return X, X[:, :k] @ (w / w.norm())


def scm_prior_tables(batch_size: int, n_rows: int, n_features: list[int], fit_rows: int, seed: int, device,
                     mlp_prob: float = 0.7, pad_features: int | None = None):
    """A batch of SCM-prior tables ``(X [B, N, F_pad], y [B, N], meta)`` (regression)."""
    rng = np.random.default_rng(seed)
    hps = [sample_hyperparams(rng, mlp_prob) for _ in range(batch_size)]
    Fpad = pad_features or max(n_features)
    X = torch.zeros(batch_size, n_rows, Fpad, device=device)
    y = torch.zeros(batch_size, n_rows, device=device)
    mlp = [i for i, h in enumerate(hps) if h.scm_type == "mlp"]
    tree = [i for i, h in enumerate(hps) if h.scm_type == "tree"]
    if mlp:
        xm, ym = mlp_scm_batch([hps[i] for i in mlp], [n_features[i] for i in mlp], n_rows, fit_rows,
                               int(rng.integers(0, 2 ** 62)), device, rng)
        X[mlp, :, : xm.shape[-1]] = xm
        y[mlp] = ym
    if tree:
        xt, yt = tree_scm_batch([hps[i] for i in tree], [n_features[i] for i in tree], n_rows, fit_rows,
                                int(rng.integers(0, 2 ** 62)), device, rng)
        X[tree, :, : xt.shape[-1]] = xt
        y[tree] = yt
    # degenerate draws (non-finite or constant context) fall back to a linear table
    fin = torch.isfinite(X[:, :fit_rows]).flatten(1).all(1) & torch.isfinite(y[:, :fit_rows]).all(1)
    var_ok = (X[:, :fit_rows].std(1, unbiased=False) > 1e-8).any(1) & (y[:, :fit_rows].std(1, unbiased=False) > 1e-8)
    bad = (~(fin & var_ok)).nonzero().flatten().tolist()
    gen = torch.Generator(device=device).manual_seed(int(rng.integers(0, 2 ** 62)))
    for b in bad:
        xb, yb = fallback_linear(n_rows, n_features[b], gen, device)
        X[b] = 0.0
        X[b, :, : n_features[b]] = xb
        y[b] = yb
    X, y = stabilize(X, y, n_features, fit_rows)
    meta = {"scm_type": [h.scm_type for h in hps], "fallback": bad, "hyper": hps}
    return X, y, meta
