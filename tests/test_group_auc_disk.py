"""Disk-backed group AUC (QAUC / UAUC): partitioned spill files against a brute-force
per-group AUC on the same score bins, evaluation through the trainer, group keys from a
Parquet column (CPU)."""

import numpy as np
import pyarrow as pa
import pytest
import torch

from mdl_b200.data.parquet import group_keys
from mdl_b200.metrics.auc import binary_auc, group_auc
from mdl_b200.metrics.group_auc_disk import DiskGroupAUC, probability_bins


def _brute(groups, logits, labels, bins):
    b = torch.from_numpy(probability_bins(logits, bins)).double()
    return group_auc(b, labels.double(), groups.tolist())


def test_matches_bruteforce_over_batches_and_partitions(tmp_path):
    g = torch.Generator().manual_seed(0)
    n, bins = 5000, 64
    groups = torch.randint(0, 300, (n,), generator=g)
    labels = (torch.rand(n, generator=g) < 0.3).double()
    logits = torch.randn(n, generator=g) + labels * 0.8 + (groups % 7).double() * 0.1
    scen = torch.randint(0, 3, (n,), generator=g)
    member = torch.nn.functional.one_hot(scen, 3).bool()
    with DiskGroupAUC(bins, partitions=7, directory=str(tmp_path / "spill")) as acc:
        for lo in range(0, n, 700):  # several batches: a group's records span batches
            sl = slice(lo, lo + 700)
            acc.add(0, groups[sl], logits[sl], labels[sl], member[sl])
            acc.add(1, groups[sl], -logits[sl], labels[sl], None)
        vals = acc.compute_all()
        assert acc.records < 2 * n * 2
    assert vals[(0, -1)] == pytest.approx(_brute(groups, logits, labels, bins), abs=1e-12)
    assert vals[(1, -1)] == pytest.approx(_brute(groups, -logits, labels, bins), abs=1e-12)
    for s in range(3):
        sel = scen == s
        assert vals[(0, s)] == pytest.approx(_brute(groups[sel], logits[sel], labels[sel], bins), abs=1e-12)
    assert (1, 0) not in vals


def test_single_class_groups_are_skipped():
    with DiskGroupAUC(16, partitions=2) as acc:
        acc.add(0, torch.tensor([1, 1, 2, 2]), torch.tensor([0.1, 0.2, -1.0, 2.0]), torch.tensor([1.0, 1.0, 0.0, 1.0]))
        # group 1 holds only positives; group 2: the positive scores above the negative
        assert acc.compute(0) == pytest.approx(1.0)
    assert binary_auc(torch.tensor([-1.0, 2.0]), torch.tensor([0.0, 1.0])) == 1.0


def test_group_keys_from_columns():
    ints = group_keys(pa.chunked_array([[5, None, 7]]))
    assert ints.tolist() == [5, -1, 7]
    text = group_keys(pa.chunked_array([["q1", "q2", None, "q1"]]))
    assert text[0] == text[3] and text[0] != text[1] and text[2] == -1 and (text[[0, 1, 3]] >= 0).all()
    again = group_keys(pa.array(["q1"]))
    assert again[0] == text[0]  # deterministic across calls


def test_evaluate_reports_qauc():
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import baseline_config
    from mdl_b200.data.synthetic import SyntheticGenerator
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.evaluate import evaluate, predict_logits
    from mdl_b200.train.trainer import Trainer

    m, spec = baseline_config(1)
    cfg = app_config_from_mapping(m)
    model = build_model(cfg, device="cpu")
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batches = []
    for i in range(3):
        b = gen.batch(128)
        b.group_key = torch.arange(128) % 11 + 100 * (i % 2)
        batches.append(b)
    res = evaluate(tr, batches, bins=256, group_metric="qauc")
    assert res["qauc_records"] > 0
    # brute force over the same logits
    task = cfg.task_names[0]
    lg = torch.cat([predict_logits(tr, b)[:, 0] for b in batches])
    y = torch.cat([b.labels[:, 0] for b in batches])
    gk = torch.cat([b.group_key for b in batches])
    keep = torch.cat([b.label_mask[:, 0] > 0 if b.label_mask is not None else torch.ones(b.rows, dtype=torch.bool)
                      for b in batches])
    expect = _brute(gk[keep], lg[keep], y[keep], 256)
    assert res["qauc"][task]["all"] == pytest.approx(expect, abs=1e-9)
    with pytest.raises(ValueError, match="group_id"):
        b = gen.batch(16)
        evaluate(tr, [b], group_metric="uauc")
