"""The reference arm of bench.py on CPU: the unmodified reference (installed under
baseline/_ref) builds and trains one step of each benchmark workload it supports,
scaled down, through the harness bench.py uses. Skipped when the reference is not
installed."""

import math

import pytest
import torch

from baseline import install

pytestmark = pytest.mark.skipif(not install.installed(), reason="reference not installed under baseline/_ref")


def _step(n, **kw):
    from baseline import reference_harness as rh
    from mdl_b200.data.baseline_configs import scaled_config

    mapping, spec = scaled_config(n, 1e-4, num_fields=12, batch=32, **kw)
    mapping["runtime"]["device"] = "cpu"
    torch.manual_seed(0)
    trainer = rh.ReferenceTrainer(mapping, device=torch.device("cpu"), rank=0, world=1, local=0, cuda_graphs=False)
    batches = rh.reference_batches(trainer, mapping, spec, 32, 2)
    losses = [float(trainer.step(b)) for b in batches]
    assert all(math.isfinite(v) for v in losses), losses
    return trainer


def test_reference_rankmixer_workload_steps():
    t = _step(2)
    assert t.config.model.name == "rankmixer"


def test_reference_mdl_rankmixer_workload_steps():
    t = _step(3)
    assert t.config.model.name == "mdl_rankmixer"
    assert len(t.config.scenarios.names) == 5


def test_reference_onetrans_workload_steps():
    t = _step(4, seq_len=16, num_layers=2)
    assert t.config.model.name == "onetrans"


def test_reference_mdl_onetrans_workload_steps():
    t = _step(4, seq_len=16, num_layers=2, mdl=True)
    assert t.config.model.name == "mdl_onetrans"
