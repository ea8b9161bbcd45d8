"""Sparse-MoE per-token FFN: gate policies against a per-expert loop of the reference
semantics, the regulariser and its controller, RankMixer / MDL training with MoE
blocks, and the CUDA path against the fp32 CPU definition."""

import pytest
import torch
import torch.nn.functional as F

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.ops._ext import check_error_word
from mdl_b200.ops.moe import SparseMoEPerTokenFFN, step_moe_controllers
from mdl_b200.train.trainer import Trainer


def _looped(moe: SparseMoEPerTokenFFN, x: torch.Tensor) -> torch.Tensor:
    """Per token, per expert ``nn.Linear`` evaluation from the reference-layout tensors."""

    sd = moe.reference_state_dict("")
    outs = []
    for t in range(moe.num_tokens):
        v = x[:, t]
        sparse = torch.relu(F.linear(v, sd[f"sparse_routers.{t}.weight"], sd[f"sparse_routers.{t}.bias"]))
        experts = torch.stack([F.linear(F.gelu(F.linear(v, sd[f"experts.{t}.{e}.0.weight"], sd[f"experts.{t}.{e}.0.bias"])),
                                        sd[f"experts.{t}.{e}.3.weight"], sd[f"experts.{t}.{e}.3.bias"])
                               for e in range(moe.num_experts)], dim=1)
        if not moe.training:
            gate = sparse * (sparse > moe.inference_threshold)
        elif not moe.use_dtsi:
            gate = sparse
        else:
            dense = torch.softmax(F.linear(v, sd[f"dense_routers.{t}.weight"], sd[f"dense_routers.{t}.bias"]), -1)
            gate = dense if moe.dtsi_training_output == "dense_router" else 0.5 * (dense + sparse)
        outs.append((experts * gate.unsqueeze(-1)).sum(1))
    return torch.stack(outs, dim=1)


@pytest.mark.parametrize("kw,train", [(dict(use_dtsi=True, dtsi_training_output="dense_router"), True),
                                      (dict(use_dtsi=True, dtsi_training_output="mean"), True),
                                      (dict(use_dtsi=False), True),
                                      (dict(use_dtsi=False, inference_threshold=0.05), False)])
def test_moe_matches_per_expert_loop(kw, train):
    torch.manual_seed(0)
    moe = SparseMoEPerTokenFFN(3, 16, 24, num_experts=4, **kw)
    moe.train(train)
    x = torch.randn(5, 3, 16)
    torch.testing.assert_close(moe(x), _looped(moe, x), atol=1e-5, rtol=1e-5)
    sparse = torch.relu(torch.einsum("btd,ted->bte", x, moe.sparse_router_weight) + moe.sparse_router_bias)
    torch.testing.assert_close(moe.last_regularization_loss, 1e-8 * sparse.sum(-1).mean())
    assert moe.update_pending == train


def test_controller_moves_the_coefficient():
    moe = SparseMoEPerTokenFFN(2, 8, 8, use_dtsi=False, target_active_ratio=0.25, regularization_multiplier=2.0)
    moe(torch.randn(4, 2, 8))
    moe.last_active_ratio = torch.tensor(0.5)
    step_moe_controllers([moe])
    assert moe.regularization_coefficient.item() == pytest.approx(2e-8)
    step_moe_controllers([moe])          # nothing pending until the next training forward
    assert moe.regularization_coefficient.item() == pytest.approx(2e-8)
    moe(torch.randn(4, 2, 8))
    moe.last_active_ratio = torch.tensor(0.1)
    step_moe_controllers([moe])
    assert moe.regularization_coefficient.item() == pytest.approx(1e-8)


def _cfg(n=2, **model):
    m, spec = scaled_config(n, 1e-4, num_fields=12, batch=64)
    m["runtime"]["device"] = "cpu"
    m["model"].update({"token_dim": 64, "hidden_dim": 64, "task_head_hidden_dim": 32, "num_heads": 4,
                       "rankmixer_ffn_type": "sparse_moe", "sparse_moe_num_experts": 4,
                       "sparse_moe_dtsi_training_output": "mean", "sparse_moe_regularization_initial": 1e-3})
    m["model"].update(model)
    m["tokenization"]["num_feature_tokens"] = 4
    m["training"].update({"lr_dense": 1e-3, "dense_optimizer": "adam", "lr_warmup_steps": 0})
    return app_config_from_mapping(m), spec


@pytest.mark.parametrize("n", [2, 3])
def test_moe_models_train(n):
    cfg, spec = _cfg(n)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=0)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    assert len(tr.moe) == cfg.model.num_layers
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    out = tr.forward_backward(batch)
    assert out["moe_regularization_loss"].item() > 0
    assert tr.moe[0].sparse_router_weight.grad.abs().sum() > 0
    c0 = tr.moe[0].regularization_coefficient.item()
    losses = [float(tr.train_step(batch).loss) for _ in range(10)]
    assert losses[-1] < losses[0]
    assert tr.moe[0].regularization_coefficient.item() != c0


def test_moe_reference_state_dict_names():
    cfg, _ = _cfg()
    model = build_model(cfg, device="cpu", base_seed=0)
    sd = model.reference_state_dict()
    assert sd["blocks.0.feature_ffn.experts.3.2.0.weight"].shape == (64, 64)
    assert "blocks.1.feature_ffn.dense_routers.0.bias" in sd


@pytest.mark.gpu
@pytest.mark.parametrize("n", [2, 3])
def test_moe_cuda_step_matches_cpu_reference(n):
    cfg, spec = _cfg(n)
    torch.manual_seed(0)
    cpu_model = build_model(cfg, device="cpu", base_seed=1)
    gpu_model = build_model(cfg, device="cuda", base_seed=1)
    gpu_model.load_state_dict({k: v.cuda() for k, v in cpu_model.state_dict().items()})
    gpu_model.store.slab.copy_(cpu_model.store.slab)
    cpu_tr = Trainer(cfg, cpu_model, device=torch.device("cpu"))
    gpu_tr = Trainer(cfg, gpu_model, device=torch.device("cuda"))
    batch = SyntheticGenerator(cpu_model.encoder.batch_plan, spec).batch(64)
    out_c = cpu_tr.forward_backward(batch)
    out_g = gpu_tr.forward_backward(batch.to("cuda"))
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(out_g["logits"].cpu(), out_c["logits"].detach(), atol=6e-2, rtol=6e-2)
    gc, gg = cpu_tr.dense.grad, gpu_tr.dense.grad.cpu()
    scale = gc.norm().item()
    for name in cpu_tr.dense.names:
        o = cpu_tr.dense.offsets[name]
        k = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + k], gg[o:o + k]
        err = (ref - got).norm().item()
        assert err <= 0.08 * ref.norm().item() + 2e-3 * scale, (name, err, ref.norm().item())
