"""Loss reductions of the training step against the reference's definitions
(``_loss_terms_from_batch``, ``src/train.py:5890-6031``), written out here in plain
PyTorch: ``sum``, ``mean_per_task`` and ``mean_per_request_per_task`` (per-request
means over candidates, then the mean over requests with a labelled candidate)."""

import copy

import pytest
import torch
import torch.nn.functional as F

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config
from mdl_b200.data.synthetic import SequenceSpec, FieldSpec, SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer


def _setup(reduction, cpr=4):
    m, spec = scaled_config(2, 0.0002, num_fields=8, batch=64)
    m["runtime"].update({"device": "cpu", "precision": "fp32"})
    m["model"].update({"token_dim": 64, "hidden_dim": 128, "task_head_hidden_dim": 32, "num_heads": 4})
    m["tokenization"]["num_feature_tokens"] = 4
    m["sequences"] = [{"name": "hist", "max_length": 12, "encoder": "mean_pool", "pool_dim": 16,
                       "fields": [{"name": "item", "kind": "categorical", "source": "hist_item", "embedding_dim": 8,
                                   "encoding": {"type": "identity", "max_id": 500}}]}]
    m["tokenization"]["feature_token_inputs"] = [f["name"] for f in m["features"]] + ["hist"]
    m["training"]["loss_reduction"] = reduction
    cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=0)
    spec = copy.deepcopy(spec)
    spec.sequences = {"hist": SequenceSpec(fields={"item": FieldSpec(vocab=500)}, max_len=12, min_len=1,
                                           candidates_per_request=cpr)}
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    g = torch.Generator().manual_seed(1)
    batch.label_mask = (torch.rand(batch.labels.shape, generator=g) > 0.3).float()
    return cfg, model, Trainer(cfg, model, device=torch.device("cpu")), batch


def _reference_loss(logits, labels, mask, reduction, row_indices=None):
    element = F.binary_cross_entropy_with_logits(logits, labels, reduction="none")
    if reduction == "mean_per_request_per_task":
        req, inv = torch.unique(row_indices, sorted=True, return_inverse=True)
        num = torch.zeros(req.numel(), logits.shape[1]).index_add(0, inv, element * mask)
        cnt = torch.zeros(req.numel(), logits.shape[1]).index_add(0, inv, mask)
        means = torch.where(cnt > 0, num / cnt.clamp_min(1.0), torch.zeros_like(num))
        task_num, task_cnt = means.sum(0), (cnt > 0).float().sum(0)
    else:
        task_num, task_cnt = (element * mask).sum(0), mask.sum(0)
    if reduction == "sum":
        return task_num.sum()
    return (task_num * torch.where(task_cnt > 0, 1.0 / task_cnt.clamp_min(1.0), torch.zeros_like(task_cnt))).sum()


@pytest.mark.parametrize("reduction", ["sum", "mean_per_task", "mean_per_request_per_task"])
def test_loss_matches_reference_definition(reduction):
    cfg, model, tr, batch = _setup(reduction)
    out = tr.forward_backward(batch)
    ri = batch.sequences["hist"]["row_indices"]
    want = _reference_loss(out["logits"].detach().float(), batch.labels.float(), batch.label_mask, reduction, ri)
    torch.testing.assert_close(out["loss"].detach().float(), want, rtol=1e-5, atol=1e-6)


def test_mean_per_request_needs_request_rows():
    cfg, model, tr, batch = _setup("mean_per_request_per_task", cpr=1)
    with pytest.raises(ValueError, match="row_indices"):
        tr.forward_backward(batch)


def test_request_level_sequence_work_matches_per_candidate_sequences():
    """Sequence work done once per request (request-level rows + row_indices) gives the
    same loss and gradients as the same sequences copied onto every candidate row."""

    m, spec = scaled_config(2, 0.0002, num_fields=8, batch=64)
    m["runtime"].update({"device": "cpu", "precision": "fp32"})
    m["model"].update({"token_dim": 64, "hidden_dim": 128, "task_head_hidden_dim": 32, "num_heads": 4})
    feats = [f["name"] for f in m["features"]]
    field = {"name": "item", "kind": "categorical", "source": "x_item", "embedding_dim": 8,
             "encoding": {"type": "identity", "max_id": 500}}
    age = {"name": "age", "kind": "dense", "source": "x_age", "dimension": 1}
    m["sequences"] = [
        {"name": "s_mean", "max_length": 12, "encoder": "mean_pool", "pool_dim": 16, "fields": [field]},
        {"name": "s_att", "max_length": 12, "encoder": "attention_pool", "pool_dim": 16, "fields": [field],
         "target_inputs": [feats[0]]},
        {"name": "s_longer", "max_length": 16, "encoder": "longer", "fields": [field, age], "time_delta_field": "age",
         "longer_dim": 32, "longer_num_heads": 1, "longer_query_tokens": 4, "longer_cls_tokens": 1,
         "longer_candidate_global_tokens": 1, "rankmixer_summary_tokens": 2, "target_inputs": [feats[1]],
         "longer_output": "summary"},
    ]
    m["tokenization"]["num_feature_tokens"] = 4
    m["tokenization"]["feature_token_inputs"] = feats + ["s_mean", "s_att", "s_longer"]
    cfg = app_config_from_mapping(m)
    spec = copy.deepcopy(spec)
    spec.sequences = {
        "s_mean": SequenceSpec(fields={"item": FieldSpec(vocab=500)}, max_len=12, min_len=1, candidates_per_request=4),
        "s_att": SequenceSpec(fields={"item": FieldSpec(vocab=500)}, max_len=12, min_len=1, candidates_per_request=4),
        "s_longer": SequenceSpec(fields={"item": FieldSpec(vocab=500)}, max_len=16, min_len=1, dense_width=1,
                                 candidates_per_request=4),
    }
    results = []
    for expanded in (False, True):
        torch.manual_seed(0)
        model = build_model(cfg, device="cpu", base_seed=0)
        tr = Trainer(cfg, model, device=torch.device("cpu"))
        batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
        if expanded:  # every candidate row carries its own copy of its request's events
            for seq in batch.sequences.values():
                ri = seq.pop("row_indices")
                L = seq["ids"].shape[1] // seq["lengths"].numel()
                ids = seq["ids"].view(seq["ids"].shape[0], -1, L)
                seq["ids"] = ids.index_select(1, ri).reshape(ids.shape[0], -1)
                seq["lengths"] = seq["lengths"].index_select(0, ri)
                if "dense" in seq:
                    d = seq["dense"].view(-1, L, seq["dense"].shape[1])
                    seq["dense"] = d.index_select(0, ri).reshape(-1, d.shape[2])
        out = tr.forward_backward(batch)
        results.append((float(out["loss"].detach()), tr.dense.grad.clone()))
    assert abs(results[0][0] - results[1][0]) < 1e-5, results
    torch.testing.assert_close(results[0][1], results[1][1], rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize("reduction", ["sum", "mean_per_task", "mean_per_request_per_task"])
def test_loss_matches_reference_module(reduction, weighted):
    """The training step's loss against the reference's own ``_loss_terms_from_batch`` on
    the same logits, labels, label mask, candidate-to-request map and task loss weights."""

    from baseline import install

    if not install.installed():
        pytest.skip("reference not installed under baseline/_ref")
    from baseline import reference_harness as rh

    rh._import_reference()
    from src.dataloader import FeatureBatch
    from src.train import _loss_terms_from_batch

    cfg, model, tr, batch = _setup(reduction)
    weights = None
    if weighted:
        weights = tuple(0.5 + i for i in range(len(cfg.task_names)))
        tr.task_weights = torch.tensor(weights, dtype=tr.task_weights.dtype)
    out = tr.forward_backward(batch)
    logits = out["logits"].detach().float()
    ri = batch.sequences["hist"]["row_indices"]
    ref_batch = FeatureBatch(features={"hist": {"row_indices": ri}}, labels=batch.labels.float(),
                             label_mask=batch.label_mask.float(),
                             scenario_id=torch.zeros(batch.rows, dtype=torch.long), group_id=[])
    want, _, _ = _loss_terms_from_batch({"logits": logits}, ref_batch, loss_reduction=reduction,
                                     task_loss_weights=weights)
    torch.testing.assert_close(out["loss"].detach().float(), want, rtol=1e-5, atol=1e-6)
