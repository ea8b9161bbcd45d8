"""AUC parity with the reference on identical seeded data (BASELINE workload 1: tiny
RankMixer, fp32 on CPU).

Both frameworks start from the same weights (this framework's initial dense weights
under the reference's parameter names, the same embedding tables), train 200 steps
on the same synthetic batches with the same optimizers (RMSprop on dense
parameters -- the reference's only dense optimizer --, row-wise Adagrad on the
tables), then score the same held-out batches. The reference runs unmodified from
``baseline/_ref`` through its own model, loss and optimizers; skipped when it is not
installed."""

import pytest
import torch

from baseline import install
from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import baseline_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.metrics.auc import binary_auc
from mdl_b200.models.factory import build_model
from mdl_b200.train.trainer import Trainer

pytestmark = pytest.mark.skipif(not install.installed(), reason="reference not installed under baseline/_ref")

STEPS = 200


def test_auc_matches_reference_after_200_steps():
    from baseline import reference_harness as rh

    mapping, spec = baseline_config(1)
    mapping["training"]["dense_optimizer"] = "rmsprop"
    cfg = app_config_from_mapping(mapping)
    torch.manual_seed(0)
    ours = build_model(cfg, device="cpu", base_seed=0)
    trainer = Trainer(cfg, ours, device=torch.device("cpu"))
    ref = rh.ReferenceTrainer(mapping, device=torch.device("cpu"), rank=0, world=1, local=0, cuda_graphs=False)
    # identical starting point
    missing, unexpected = ref.base.load_state_dict(ours.reference_state_dict(), strict=False)
    assert not unexpected, unexpected
    assert all(n.startswith("encoder_bank.embeddings.") for n in missing), missing
    with torch.no_grad():
        for t in ours.store.layouts:
            ref.base.encoder_bank.embeddings[t.name].weight.copy_(ours.store.weight(t.name))
    plan = ours.encoder.batch_plan
    gen = SyntheticGenerator(plan, spec)
    train = [gen.batch(256) for _ in range(STEPS)]
    held_out = [gen.batch(256) for _ in range(16)]
    ours_losses, ref_losses = [], []
    for b in train:
        ours_losses.append(float(trainer.train_step(b).loss))
        ref_losses.append(float(ref.step(rh.to_feature_batch(ref.rdata, b, plan))))
    assert abs(ours_losses[0] - ref_losses[0]) < 1e-5, (ours_losses[0], ref_losses[0])
    scores_o, scores_r, labels = [], [], []
    ref.model.eval()
    with torch.no_grad():
        for b in held_out:
            scores_o.append(trainer.predict_logits(b)[:, 0].float())
            fb = rh.to_feature_batch(ref.rdata, b, plan)
            scores_r.append(ref.model(fb.features, fb.scenario_id)["logits"][:, 0].float())
            labels.append(b.labels[:, 0])
    y = torch.cat(labels)
    auc_o = binary_auc(torch.cat(scores_o), y)
    auc_r = binary_auc(torch.cat(scores_r), y)
    assert auc_o > 0.55, auc_o  # the model learned something
    print(f"AUC ours {auc_o:.6f} reference {auc_r:.6f} final loss ours {ours_losses[-1]:.6f} reference {ref_losses[-1]:.6f}")
    assert abs(auc_o - auc_r) <= 1e-3, (auc_o, auc_r)


def test_auc_matches_reference_gloo_two_ranks(tmp_path):
    """The same comparison at world size 2 (gloo ranks on CPU): both frameworks shard
    their tables over the two ranks, each rank trains on its half of every union
    batch, and the AUC over both ranks' held-out scores is compared."""

    import json
    import time

    import torch.multiprocessing as mp

    from baseline.reference_harness import auc_parity_worker

    out = str(tmp_path / "auc.json")
    ctx = mp.start_processes(auc_parity_worker, args=(2, str(tmp_path / "pg"), out, STEPS),
                             nprocs=2, join=False, start_method="spawn")
    deadline = time.monotonic() + 600
    while not ctx.join(timeout=5):
        if time.monotonic() > deadline:
            for proc in ctx.processes:
                if proc.is_alive():
                    proc.kill()
            pytest.fail("parity ranks did not finish within 600 s")
    with open(out) as fh:
        r = json.load(fh)
    print(r)
    assert abs(r["first_loss"][0] - r["first_loss"][1]) < 1e-4, r
    assert r["auc_ours"] > 0.55, r
    assert abs(r["auc_ours"] - r["auc_reference"]) <= 1e-3, r
