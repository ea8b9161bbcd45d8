"""Every config the reference ships builds here and trains one step on CPU.

The reference's ``configs/*.yaml`` load unchanged through this framework's loader;
``shrink_mapping`` then caps table rows, sequence lengths, the batch and the FFN
hidden widths (the architecture stays as configured: feature groups, sequence
encoders, token layout, model family and token widths), and one training step runs
on synthetic data of that shape. Skipped when the reference sources are not available."""

import math
import os

import pytest
import torch

from baseline.install import reference_source
from mdl_b200.config import app_config_from_mapping, load_config_mapping
from mdl_b200.config.scale import shrink_mapping

CONFIG_DIR = os.path.join(reference_source(), "configs")
NAMES = sorted(f[:-5] for f in os.listdir(CONFIG_DIR) if f.endswith(".yaml")) if os.path.isdir(CONFIG_DIR) else []

pytestmark = pytest.mark.skipif(not NAMES, reason="reference configs not available")


@pytest.mark.parametrize("name", NAMES)
def test_reference_config_builds_and_trains_one_step(name):
    from mdl_b200.data.synthetic import SyntheticGenerator, synthetic_spec_from_config
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    mapping = shrink_mapping(load_config_mapping(os.path.join(CONFIG_DIR, f"{name}.yaml")), batch=8,
                             max_hidden=256)
    cfg = app_config_from_mapping(mapping)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=0)
    enc = model.encoder
    seqs = [s for s in cfg.sequences if s.name in enc.seq_plans]
    spec = synthetic_spec_from_config(cfg, enc.batch_plan, sequences=seqs)
    batch = SyntheticGenerator(enc.batch_plan, spec).batch(8)
    trainer = Trainer(cfg, model, device=torch.device("cpu"))
    loss = float(trainer.train_step(batch).loss)
    assert math.isfinite(loss) and loss > 0
    # every sequence the config feeds into tokens is encoded (nothing dropped silently)
    used = set(cfg.resolved.tokenization.feature_token_inputs)
    for tok in (*cfg.resolved.tokenization.scenario_token_specs, *cfg.resolved.tokenization.task_token_specs):
        used |= set(tok.resolved_inputs())
    for s in cfg.sequences:
        if s.name in used and s.encoder != "raw":
            assert s.name in enc.summary_names, f"sequence {s.name} ({s.encoder}) is not encoded"
