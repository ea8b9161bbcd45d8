"""MDL (mdl_rankmixer) model on CPU: construction of every variant, token layout,
training progress, and the masking semantics of scenario pooling."""

import pytest
import torch

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config, scaled_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer


def _cfg(**model):
    m, spec = scaled_config(3, 0.0001, num_fields=24, batch=64)
    m["runtime"]["device"] = "cpu"
    m["model"].update({"token_dim": 64, "hidden_dim": 128, "task_head_hidden_dim": 32, "num_heads": 4})
    m["model"].update(model)
    m["tokenization"]["num_feature_tokens"] = 8
    m["training"].update({"lr_dense": 1e-3, "dense_optimizer": "adam", "lr_warmup_steps": 0})
    return app_config_from_mapping(m), spec


def test_config3_resolves():
    m, spec = baseline_config(3)
    cfg = app_config_from_mapping(m)
    res = cfg.resolved.tokenization
    assert len(res.scenario_token_specs) == 5 * 4 + 1
    assert [t.name for t in res.task_token_specs] == ["click", "like", "finish"]
    # scenario/task-scope features are not feature-token inputs
    assert "scene_id" not in res.feature_token_inputs
    assert "prior_click" not in res.feature_token_inputs
    assert spec.task_rates == [0.08, 0.02, 0.3]


def test_batch_layout_covers_domain_inputs():
    cfg, spec = _cfg()
    model = build_model(cfg, device="cpu", base_seed=0)
    enc = model.encoder
    assert enc.batch_names[: len(enc.inputs)] == enc.inputs
    assert set(enc.batch_names[len(enc.inputs):]) == ({"scene_id", "prior_click", "prior_like", "prior_finish"}
                                                      | {f"prior_scene{i}" for i in range(5)})
    assert model.Ns == 21 and model.Nt == 3
    # the scene id feature carries scenario_id + 1
    batch = SyntheticGenerator(enc.batch_plan, spec).batch(32)
    si = enc.batch_names.index("scene_id")
    ids = batch.ids[batch.offsets[si * 32]:batch.offsets[(si + 1) * 32]]
    assert torch.equal(ids, batch.scenario_id + 1)


@pytest.mark.parametrize("variant", [
    {},
    {"mdl_token_state": "split", "scene_feature_bias": "none"},
    {"use_scenario_tokens": False, "scene_feature_bias": "none"},
    {"use_task_tokens": False},
    {"use_scenario_feature_interaction": False, "use_task_feature_interaction": False},
    {"mdl_feature_interaction": "direct_ffn", "scene_feature_bias": "additive"},
    {"use_global_scenario_token": False, "tokens_per_scenario": 1},
])
def test_variants_train(variant):
    cfg, spec = _cfg(**variant)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=0)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batches = [SyntheticGenerator(model.encoder.batch_plan, spec).batch(64) for _ in range(2)]
    first = float(tr.train_step(batches[0]).loss)
    for i in range(15):
        last = float(tr.train_step(batches[i % 2]).loss)
    assert last < first


def test_inactive_scene_tokens_get_no_gradient():
    """Only the active scene's tokens (and the global token) reach the loss."""

    cfg, spec = _cfg()
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=0)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    batch.scenario_id.fill_(2)
    # the scene id feature mirrors scenario_id
    si = model.encoder.batch_names.index("scene_id")
    batch.ids[batch.offsets[si * 64]:batch.offsets[(si + 1) * 64]] = 3
    tr.forward_backward(batch)
    g = model.blocks[0].scenario_ffn.output_weight.grad  # [Ns, D, H]
    tps = model.tps
    active = set(range(2 * tps, 3 * tps)) | {model.Ns - 1}
    for tok in range(model.Ns):
        nz = g[tok].abs().max().item() > 0
        assert nz == (tok in active), tok
