"""Human-readable training log lines and the environment record (CPU)."""

import json
import math

import torch

from mdl_b200.train.train_log import TrainLog, environment, environment_line


class _Res:
    def __init__(self, logits):
        self.logits = logits


class _Batch:
    def __init__(self, labels, mask=None):
        self.labels, self.label_mask, self.rows = labels, mask, labels.shape[0]


def test_window_lines_and_collapse_warning():
    log = TrainLog(["click", "like"], world=2, micro_batches=1, checkpoint_every=100)
    lg = torch.tensor([[0.0, 4.0], [2.0, 4.0], [-2.0, 4.0]])
    y = torch.tensor([[0.0, 1.0], [1.0, 1.0], [0.0, 1.0]])
    log.step(_Res(lg), _Batch(y), wait_s=0.25)
    log.step(_Res(lg), _Batch(y, torch.tensor([[1.0, 0.0], [1.0, 0.0], [1.0, 0.0]])), wait_s=0.25)
    lines = log.lines(step=10, loss=0.5, sparse_rows=7)
    assert lines[0].startswith("Train step | step=10 | logloss=0.500000 active_ranks=2/2")
    assert "local_rows=6" in lines[0] and "dataloader_wait_s=0.5000" in lines[0]
    assert "sparse_local_rows=7" in lines[0] and "checkpoint=on(every=100)" in lines[0]
    click = next(l for l in lines if l.startswith("Train task | step=10 task=click"))
    bce = torch.nn.functional.binary_cross_entropy_with_logits(lg[:, 0], y[:, 0]).item()
    assert f"logloss={bce:.6f}" in click
    mean = lg[:, 0].mean().item()
    std = math.sqrt((lg[:, 0] ** 2).mean().item() - mean ** 2)
    assert f"logit_mean={mean:.6f}" in click and f"logit_std={std:.6f}" in click
    # "like" saw 3 masked-in rows with p = sigmoid(4) = 0.982 > 0.9: collapse warning
    assert any(l.startswith("Train task warning | step=10 task=like") for l in lines)
    # the window resets
    assert log.lines(step=11, loss=None)[0].startswith("Train step | step=11 | logloss=none")


def test_environment_record():
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import baseline_config

    m, _ = baseline_config(1)
    env = environment(app_config_from_mapping(m), world=1, device=torch.device("cpu"))
    assert env["torch"] == torch.__version__ and env["world_size"] == 1 and env["model"]
    line = environment_line(env)
    assert line.startswith("Environment | ") and json.loads(line[len("Environment | "):])["world_size"] == 1


def test_cli_train_prints_stable_prefixes():
    import subprocess
    import sys

    out = subprocess.run([sys.executable, "-m", "mdl_b200", "train", "--benchmark-config", "1", "--synthetic",
                          "--max-steps", "4", "--log-every", "2", "--set", "training.batch_size=64"],
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.splitlines()
    assert lines[0].startswith("Environment | ")
    steps = [l for l in lines if l.startswith("Train step | ")]
    assert [l.split()[3] for l in steps] == ["step=2", "step=4"]
    assert any(l.startswith("Train task | step=4 task=") for l in lines)


def test_train_from_host_matches_train_step():
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import baseline_config
    from mdl_b200.data.synthetic import SyntheticGenerator
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    m, spec = baseline_config(1)
    cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batches = [gen.batch(64) for _ in range(3)]
    a = Trainer(cfg, model, device=torch.device("cpu"))
    losses = torch.zeros(3)
    assert a.train_from_host(iter(batches), loss_out=losses) == 3 and a.step_index == 3
    torch.manual_seed(0)
    model2 = build_model(cfg, device="cpu", base_seed=1)
    b = Trainer(cfg, model2, device=torch.device("cpu"))
    ref = [float(b.train_step(x).loss) for x in batches]
    torch.testing.assert_close(losses, torch.tensor(ref))
