"""``NoriCausal``: causal structure of one observational table (reference
``causal/estimator.py:67-265``).

Modes (same semantics as the reference): ``"target"`` one target-aware pass with ``y``
in the target slot; ``"null"`` one pass with a learned null target token;
``"subgraph"`` ``n_subsets`` random column subsets of at most ``window`` columns, each
read once with its last column in the target slot, logits averaged per pair;
``"auto"`` picks ``target`` (with ``y`` and at most ``target_max_features`` features),
target-anchored subgraph voting (wider tables: ``y`` takes the target slot of every
subset containing it, then subsets of ``y`` plus its least-covered features are added
until each feature shared ``min_target_coverage`` subsets with ``y``) or ``subgraph``
(no ``y``).  Pairs never sampled together get logit -20.  ``threshold`` decodes a 0/1
graph keeping the stronger direction of two-cycles (exact ties keep i -> j for i < j).
"""

from __future__ import annotations

import numpy as np
import torch

try:
    from sklearn.base import BaseEstimator
except ImportError:  # pragma: no cover
    BaseEstimator = object

UNCOVERED_LOGIT = -20.0
_NETWORKS: dict = {}


def get_decoded_graph(prob: np.ndarray, threshold: float) -> np.ndarray:
    p = np.asarray(prob, np.float64)
    g = p > float(threshold)
    np.fill_diagonal(g, False)
    both = g & g.T
    g &= ~(both & (p < p.T))
    g &= ~np.tril(both & (p == p.T))
    return g.astype(np.uint8)


class NoriCausal(BaseEstimator):
    def __init__(self, *, model="noricausal-31m", checkpoint=None, network=None, mode="auto", target_max_features=25,
                 n_subsets=64, window=30, min_target_coverage=3, threshold=None, device="auto", random_state=0):
        self.model = model
        self.checkpoint = checkpoint
        self.network = network
        self.mode = mode
        self.target_max_features = target_max_features
        self.n_subsets = n_subsets
        self.window = window
        self.min_target_coverage = min_target_coverage
        self.threshold = threshold
        self.device = device
        self.random_state = random_state

    def _network(self, device):
        if self.network is not None:
            return self.network.to(device).eval(), None
        from synthefy_nori_b200.causal.network import NoriCausalNetwork
        from synthefy_nori_b200.causal.registry import resolve_causal_checkpoint

        path, thr = resolve_causal_checkpoint(self.model, self.checkpoint)
        key = (str(path), str(device))
        if key not in _NETWORKS:
            _NETWORKS[key] = NoriCausalNetwork.from_checkpoint(path, device)[0]
        return _NETWORKS[key], thr

    def fit(self, X, y=None, feature_names=None, target_name="target"):
        if self.mode not in ("auto", "subgraph", "target", "null"):
            raise ValueError(f"mode must be 'auto', 'subgraph', 'target' or 'null', got {self.mode!r}")
        if self.mode == "target" and y is None:
            raise ValueError("mode='target' needs y")
        if feature_names is None and hasattr(X, "columns"):
            feature_names = [str(c) for c in X.columns]
        X = np.asarray(X, np.float32)
        if X.ndim != 2 or X.shape[1] < 1:
            raise ValueError(f"X must be 2-D with at least one column, got {X.shape}")
        names = list(feature_names) if feature_names is not None else [f"f{j}" for j in range(X.shape[1])]
        table = X if y is None else np.column_stack([X, np.asarray(y, np.float32).reshape(-1)])
        if y is not None:
            names.append(target_name)
        if table.shape[1] < 2:
            raise ValueError("need at least two variables (columns of X plus y)")
        device = ("cuda" if torch.cuda.is_available() else "cpu") if self.device == "auto" else self.device
        net, calibrated = self._network(device)
        rng = np.random.default_rng(self.random_state)

        @torch.no_grad()
        def one_pass(cols: np.ndarray, null: bool) -> np.ndarray:
            if null:
                ph = np.random.default_rng(0).standard_normal(len(cols)).astype(np.float32)
                lg = net(torch.as_tensor(cols, device=device), torch.as_tensor(ph, device=device), null_target=True)
                return lg.cpu().numpy()[: cols.shape[1], : cols.shape[1]]
            return net(torch.as_tensor(np.ascontiguousarray(cols[:, :-1]), device=device),
                       torch.as_tensor(np.ascontiguousarray(cols[:, -1]), device=device)).cpu().numpy()

        T = table.shape[1]
        tgt = T - 1 if y is not None else None
        mode = self.mode
        if mode == "auto":
            mode = "subgraph" if tgt is None else ("target" if X.shape[1] <= self.target_max_features
                                                   else "target_subgraph")
        self.mode_ = mode
        if mode in ("null", "target"):
            logits = one_pass(table, mode == "null")
            self.pair_coverage_ = np.ones((T, T), np.int64)
        else:
            w = min(max(int(self.window), 2), T)
            acc, cnt = np.zeros((T, T)), np.zeros((T, T), np.int64)

            def add(sub):
                acc[np.ix_(sub, sub)] += one_pass(table[:, sub], False)
                cnt[np.ix_(sub, sub)] += 1

            for _ in range(int(self.n_subsets)):
                sub = rng.permutation(T)[:w]
                if mode == "target_subgraph" and tgt in sub:
                    sub = np.append(sub[sub != tgt], tgt)
                add(sub)
            if mode == "target_subgraph":
                feats = np.arange(T - 1)
                while (cov := cnt[feats, tgt]).min() < int(self.min_target_coverage):
                    least = np.lexsort((rng.random(len(feats)), cov))[: w - 1]
                    add(np.append(feats[least], tgt))
            logits = np.where(cnt > 0, acc / np.maximum(cnt, 1), UNCOVERED_LOGIT)
            self.pair_coverage_ = cnt
        logits = np.asarray(logits, np.float64)
        np.fill_diagonal(logits, 0.0)
        prob = 1.0 / (1.0 + np.exp(-np.clip(logits, -80, 80)))
        np.fill_diagonal(prob, 0.0)
        self.node_names_, self.target_index_ = names, tgt
        self.logits_, self.adjacency_ = logits, prob
        self.n_rows_, self.device_ = len(table), device
        if self.threshold is None:
            self.threshold_, self.graph_, self.edges_ = None, None, []
            return self
        thr = calibrated if self.threshold == "calibrated" else float(self.threshold)
        if thr is None:
            raise ValueError("threshold='calibrated' needs a registry model; pass a float threshold")
        self.threshold_ = float(thr)
        self.graph_ = get_decoded_graph(prob, thr)
        self.edges_ = sorted(({"source": names[i], "target": names[j], "probability": float(prob[i, j])}
                              for i, j in zip(*np.nonzero(self.graph_))), key=lambda e: -e["probability"])
        return self

    def _idx(self, node) -> int:
        if getattr(self, "graph_", None) is None:
            raise ValueError("fitted with threshold=None: no graph; read adjacency_ instead")
        return node if isinstance(node, (int, np.integer)) else self.node_names_.index(node)

    def parents(self, node) -> list:
        c = self._idx(node)
        ps = np.nonzero(self.graph_[:, c])[0]
        return [self.node_names_[i] for i in ps[np.argsort(-self.adjacency_[ps, c])]]

    def children(self, node) -> list:
        p = self._idx(node)
        cs = np.nonzero(self.graph_[p])[0]
        return [self.node_names_[j] for j in cs[np.argsort(-self.adjacency_[p, cs])]]

    def to_frame(self):
        import pandas as pd

        return pd.DataFrame(self.adjacency_, index=self.node_names_, columns=self.node_names_)
