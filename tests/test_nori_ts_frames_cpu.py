"""Nori-TS panel frames: construction, panel facts, slicing, horizon generation and the
train / horizon feature transformer."""

import numpy as np
import pandas as pd
import pytest

from synthefy_nori_b200.nori_ts import RunningIndexFeature, default_features
from synthefy_nori_b200.nori_ts.frames import (AdditionalCalendarFeature, FeatureTransformer, TimeSeriesDataFrame,
                                               generate_test_X)


def _flat():
    rows = []
    for item, n in (("a", 10), ("b", 7)):
        ts = pd.date_range("2024-01-01", periods=n, freq="h")
        rows.append(pd.DataFrame({"item_id": item, "timestamp": ts, "target": np.arange(n, dtype=float)}))
    return pd.concat(rows)


def test_construction_and_panel_facts():
    tsdf = TimeSeriesDataFrame.from_data_frame(_flat())
    assert list(tsdf.index.names) == ["item_id", "timestamp"]
    assert tsdf.num_items == 2 and list(tsdf.item_ids) == ["a", "b"]
    assert tsdf.num_timesteps_per_item().to_dict() == {"a": 10, "b": 7}
    assert tsdf.freq == "h"
    recs = TimeSeriesDataFrame.from_iterable_dataset([{"target": [1, 2, 3], "start": "2024-01-01", "freq": "D"},
                                                      {"target": [4, 5], "start": pd.Period("2024-02-01", "D")}])
    assert recs.num_items == 2 and len(recs) == 5


def test_slicing_split_and_fill():
    tsdf = TimeSeriesDataFrame.from_data_frame(_flat())
    head = tsdf.slice_by_timestep(None, -3)
    assert head.num_timesteps_per_item().to_dict() == {"a": 7, "b": 4}
    tail = tsdf.slice_by_timestep(-2, None)
    assert tail["target"].tolist() == [8.0, 9.0, 5.0, 6.0]
    train, full = tsdf.train_test_split(3)
    assert len(train) == len(tsdf) - 6 and len(full) == len(tsdf)
    before, after = tsdf.split_by_time("2024-01-01 05:00")
    assert len(before) == 10 and len(after) == 7
    gappy = tsdf.copy()
    gappy.iloc[[0, 4, 12], 0] = np.nan
    filled = TimeSeriesDataFrame(gappy).fill_missing_values()
    assert not filled["target"].isna().any()
    assert filled["target"].iloc[0] == 1.0  # leading gap back-filled within the item
    assert len(TimeSeriesDataFrame(gappy).dropna()) == len(tsdf) - 3


def test_generate_test_X_and_transformer():
    tsdf = TimeSeriesDataFrame.from_data_frame(_flat())
    test = generate_test_X(tsdf, 4)
    assert test.num_timesteps_per_item().to_dict() == {"a": 4, "b": 4}
    assert test["target"].isna().all()
    assert test.xs("b", level="item_id").index[0] == pd.Timestamp("2024-01-01 07:00")
    with pytest.raises(ValueError):
        generate_test_X(TimeSeriesDataFrame(tsdf.iloc[[0, 2, 3, 7]]), 2)  # irregular: needs freq=
    ft = FeatureTransformer(default_features())
    tr, te = ft.transform(tsdf, test)
    assert len(tr) == len(tsdf) and len(te) == 8
    assert "running_index" in tr and te["running_index"].tolist()[:4] == [10, 11, 12, 13]
    assert tr["running_index"].dtype != np.float64
    cal = AdditionalCalendarFeature(additional_seasonal_features={"hour_of_day": [12]})
    tr2, _ = FeatureTransformer([RunningIndexFeature(), cal]).transform(tsdf, test)
    assert {"hour_of_day_sin_0", "hour_of_day_sin_1"} <= set(tr2.columns)
