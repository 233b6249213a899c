"""Analysis of evaluation results (reference ``evaluation/analysis.py``).

``EvalAnalyzer`` takes the runner's ``results.csv`` (one row per model x dataset) and
answers the usual questions: per-model means / medians of every metric, the same per
source (benchmark suite), a per-dataset table of one metric, head-to-head win / tie /
loss counts and the mean difference, a pairwise win-rate matrix, checkpoint progress
for a family of labels, latency summaries (also by table size), and each dataset's
best other model next to a focus model.  Reports come out as text or Markdown; figures
are drawn with matplotlib when it is installed.
"""

from __future__ import annotations

import os
import re

import numpy as np
import pandas as pd

LOWER_IS_BETTER = ("rmse", "mae", "latency_ms")


def higher_is_better(metric: str) -> bool:
    return metric not in LOWER_IS_BETTER


class EvalAnalyzer:
    def __init__(self, results: pd.DataFrame):
        df = results.copy()
        if "error" in df:
            df = df[df["error"].isna() | (df["error"] == "")]
        self.df = df.reset_index(drop=True)

    @classmethod
    def from_csv(cls, *paths: str) -> "EvalAnalyzer":
        return cls(pd.concat([pd.read_csv(p) for p in paths], ignore_index=True))

    @classmethod
    def merge(cls, *analyzers: "EvalAnalyzer") -> "EvalAnalyzer":
        return cls(pd.concat([a.df for a in analyzers], ignore_index=True))

    @property
    def models(self) -> list[str]:
        return sorted(self.df["model"].unique())

    def metric_columns(self) -> list[str]:
        return [c for c in ("r2", "rmse", "mae") if c in self.df]

    # ------------------------------------------------------------------ tables
    def summary_by_model(self) -> pd.DataFrame:
        agg = {f"mean_{m}": (m, "mean") for m in self.metric_columns()}
        agg.update({f"median_{m}": (m, "median") for m in self.metric_columns()})
        agg["n_datasets"] = ("dataset", "nunique")
        if "latency_ms" in self.df:
            agg["total_latency_s"] = ("latency_ms", lambda s: s.sum() / 1e3)
        return self.df.groupby("model").agg(**agg).sort_values(f"mean_{self.metric_columns()[0]}",
                                                               ascending=not higher_is_better(self.metric_columns()[0]))

    def summary_by_source(self, metric: str = "r2") -> pd.DataFrame:
        return self.df.pivot_table(index="source", columns="model", values=metric, aggfunc="mean")

    def per_dataset_table(self, metric: str = "r2") -> pd.DataFrame:
        return self.df.pivot_table(index=["source", "dataset"], columns="model", values=metric, aggfunc="mean")

    def head_to_head(self, a: str, b: str, metric: str = "r2", tie: float = 1e-4) -> dict:
        t = self.per_dataset_table(metric)[[a, b]].dropna()
        d = t[a] - t[b]
        if not higher_is_better(metric):
            d = -d
        return {"model_a": a, "model_b": b, "metric": metric, "n": int(len(d)), "wins": int((d > tie).sum()),
                "ties": int((d.abs() <= tie).sum()), "losses": int((d < -tie).sum()),
                "mean_diff": float(d.mean()) if len(d) else float("nan"),
                "median_diff": float(d.median()) if len(d) else float("nan")}

    def pairwise_comparison(self, metric: str = "r2", tie: float = 1e-4) -> pd.DataFrame:
        """Share of shared datasets on which the row model beats the column model."""
        ms = self.models
        out = pd.DataFrame(np.nan, index=ms, columns=ms)
        for a in ms:
            for b in ms:
                if a != b:
                    h = self.head_to_head(a, b, metric, tie)
                    out.loc[a, b] = h["wins"] / h["n"] if h["n"] else np.nan
        return out

    def checkpoint_progression(self, prefix: str, metric: str = "r2") -> pd.DataFrame:
        """Mean metric of every model label ``<prefix>...<step>``, ordered by its step."""
        rows = []
        for m in self.models:
            if m.startswith(prefix):
                nums = re.findall(r"(\d+)", m[len(prefix):])
                rows.append({"model": m, "step": int(nums[-1]) if nums else -1,
                             f"mean_{metric}": float(self.df[self.df["model"] == m][metric].mean())})
        return pd.DataFrame(rows).sort_values("step").reset_index(drop=True) if rows else pd.DataFrame()

    def latency_summary(self) -> pd.DataFrame:
        return self.df.groupby("model")["latency_ms"].describe(percentiles=[0.5, 0.9])

    def latency_by_size(self, bins=(0, 1_000, 10_000, 100_000, np.inf)) -> pd.DataFrame:
        size = self.df["n_train"] * self.df["n_features"].clip(lower=1)
        cut = pd.cut(size, bins=list(bins), right=False)
        return self.df.assign(size_bucket=cut).pivot_table(index="size_bucket", columns="model", values="latency_ms",
                                                            aggfunc="median", observed=False)

    def comparison_vs_best_other(self, focus: str, metric: str = "r2") -> pd.DataFrame:
        t = self.per_dataset_table(metric)
        others = [c for c in t.columns if c != focus]
        if focus not in t or not others:
            return pd.DataFrame()
        best = t[others].max(axis=1) if higher_is_better(metric) else t[others].min(axis=1)
        who = t[others].idxmax(axis=1) if higher_is_better(metric) else t[others].idxmin(axis=1)
        out = pd.DataFrame({focus: t[focus], "best_other": best, "best_other_model": who})
        out["delta"] = (out[focus] - out["best_other"]) * (1 if higher_is_better(metric) else -1)
        return out.sort_values("delta")

    # ------------------------------------------------------------------ reports
    def report(self) -> str:
        lines = ["Per-model summary", self.summary_by_model().to_string(), ""]
        if "source" in self.df and self.df["source"].nunique() > 1:
            lines += ["Mean R^2 per source", self.summary_by_source().to_string(), ""]
        if len(self.models) > 1:
            lines += ["Pairwise win rate (row beats column)", self.pairwise_comparison().round(3).to_string(), ""]
        return "\n".join(lines)

    def markdown_report(self, path: str | None = None, focus: str | None = None) -> str:
        md = ["# Evaluation report", "", "## Per-model summary", "", self.summary_by_model().round(4).to_markdown(), ""]
        if "source" in self.df and self.df["source"].nunique() > 1:
            md += ["## Mean R² per source", "", self.summary_by_source().round(4).to_markdown(), ""]
        if focus is not None:
            comp = self.comparison_vs_best_other(focus)
            if not comp.empty:
                md += [f"## {focus} against the best other model per dataset", "", comp.round(4).to_markdown(), ""]
        md += ["## Per dataset (R²)", "", self.per_dataset_table().round(4).to_markdown(), ""]
        text = "\n".join(md)
        if path:
            with open(path, "w") as f:
                f.write(text)
        return text

    def plot_leaderboard(self, output_path: str, metric: str = "r2") -> str | None:
        """Bar chart of the per-model mean (needs matplotlib; returns None without it)."""
        try:
            import matplotlib

            matplotlib.use("Agg")
            import matplotlib.pyplot as plt
        except ImportError:
            return None
        s = self.df.groupby("model")[metric].agg(["mean", "sem"]).sort_values("mean")
        fig, ax = plt.subplots(figsize=(7, 0.4 * len(s) + 1.5))
        ax.barh(s.index, s["mean"], xerr=s["sem"])
        ax.set_xlabel(metric)
        fig.tight_layout()
        os.makedirs(os.path.dirname(os.path.abspath(output_path)) or ".", exist_ok=True)
        fig.savefig(output_path, dpi=120)
        plt.close(fig)
        return output_path
