"""LONGER (cross + self blocks, global tokens) and MixFormer (blocks, head): CPU training,
exact HeadMixing, and the CUDA path against the fp32 CPU definition."""

import pytest
import torch

from mdl_b200.config.loader import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.models.mixformer import head_mixing
from mdl_b200.ops._ext import check_error_word
from mdl_b200.train.trainer import Trainer


def _longer(head="none", seq_len=80, min_len=10, R=16, d=64, heads=2):
    m, spec = scaled_config(5, 1e-4, num_fields=12, batch=64, seq_len=seq_len, min_len=min_len, query_tokens=R,
                            self_layers=1, d=d, heads=heads, sequence_head=head, ns_tokens=4)
    m["model"].update({"token_dim": 16, "hidden_dim": 64, "task_head_hidden_dim": 32})
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    return app_config_from_mapping(m), spec


def _mixformer():
    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=2)
    m["model"].update({"name": "mixformer", "token_dim": 16, "hidden_dim": 64, "num_ns_tokens": 4,
                       "task_head_hidden_dim": 32})
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences["behavior"].min_len = 10
    return app_config_from_mapping(m), spec


def _mdl_mixformer(**model):
    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=2, mdl=True)
    m["model"].update({"name": "mdl_mixformer", "experimental_model_acknowledged": True, "token_dim": 32,
                       "hidden_dim": 64, "num_ns_tokens": 4, "num_heads": 2, "task_head_hidden_dim": 32})
    m["model"].update(model)
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences["behavior"].min_len = 10
    return app_config_from_mapping(m), spec


def test_head_mixing_user_heads_decoupling():
    """User heads keep only the chunks of user heads (UI-MixFormer mask)."""

    x = torch.randn(2, 4, 8)
    y = head_mixing(x, user_heads=1)
    full = head_mixing(x)
    assert torch.equal(y[:, 1:], full[:, 1:])
    assert torch.equal(y[:, 0, :2], full[:, 0, :2]) and not y[:, 0, 2:].any()


@pytest.mark.parametrize("variant", [dict(), dict(mdl_token_state="split"),
                                     dict(mdl_mixformer_query_conditioning=False, scene_feature_bias="additive"),
                                     dict(mixformer_user_head_count=1, use_task_tokens=False)])
def test_mdl_mixformer_trains_on_cpu(variant):
    cfg, spec = _mdl_mixformer(**variant)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    assert type(model).__name__ == "MDLMixFormerModel"
    assert (model.blocks[0].query_router is not None) == cfg.model.mdl_mixformer_query_conditioning
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    assert tr.forward_backward(batch)["logits"].shape == (64, 3)
    losses = [float(tr.train_step(batch).loss) for _ in range(8)]
    assert losses[-1] < losses[0]


def test_query_router_starts_as_identity():
    from mdl_b200.models.mixformer import ScenarioQueryRouter

    r = ScenarioQueryRouter(4, 16)
    q = torch.randn(3, 4, 16)
    torch.testing.assert_close(r(q, torch.randn(3, 16), native=False), q)


def test_head_mixing_is_the_chunk_transpose():
    x = torch.arange(2 * 4 * 8, dtype=torch.float32).view(2, 4, 8)
    y = head_mixing(x)
    for n in range(4):
        for m in range(4):
            assert torch.equal(y[:, n, m * 2:(m + 1) * 2], x[:, m, n * 2:(n + 1) * 2])


@pytest.mark.parametrize("make", [lambda: _longer("none"), lambda: _longer("mixformer"), _mixformer])
def test_trains_on_cpu(make):
    cfg, spec = make()
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    losses = [float(tr.train_step(batch).loss) for _ in range(6)]
    assert losses[-1] < losses[0]


@pytest.mark.gpu
@pytest.mark.parametrize("make", [lambda: _longer("none"), lambda: _longer("none", seq_len=300, min_len=50, R=130),
                                  lambda: _longer("mixformer"), _mixformer, _mdl_mixformer])
def test_cuda_step_matches_cpu_reference(make):
    cfg, spec = make()
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
    torch.testing.assert_close(out_g["loss"].cpu(), out_c["loss"].detach(), atol=3e-2, rtol=3e-2)
    gc, gg = cpu_tr.dense.grad, gpu_tr.dense.grad.cpu()
    errors = {}
    for name in cpu_tr.dense.names:
        o = cpu_tr.dense.offsets[name]
        n = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + n], gg[o:o + n]
        errors[name] = (((ref - got).norm() / (ref.norm() + 1e-9)).item(), ref.norm().item())
    # bf16 attention backward on near-uniform random-init attention: the query-path
    # gradients are ~1e-3 of the others, so they are judged against the overall scale
    scale = max(v[1] for v in errors.values())
    bad = {k: v for k, v in errors.items() if v[0] >= 0.08 and v[0] * v[1] >= 1e-3 * scale}
    assert not bad, f"grad errors (relative, reference norm): {bad}"
    ref = cpu_model.store.grad
    got = gpu_model.store.grad.cpu()
    assert ((ref - got).norm() / (ref.norm() + 1e-9)) < 0.08


def _stca_rankmixer():
    """A small RankMixer whose feature tokens include an STCA-encoded behaviour sequence."""

    m, spec = scaled_config(2, 1e-4, num_fields=12, batch=64)
    from mdl_b200.data.synthetic import FieldSpec, SequenceSpec

    m["features"].append({"name": "target_item", "kind": "categorical", "source": "target_item", "embedding_dim": 16,
                          "encoding": {"type": "identity", "max_id": 500}})
    spec.fields["target_item"] = FieldSpec(vocab=500)
    m["sequences"] = [{"name": "clicks", "max_length": 30, "encoder": "stca", "target_inputs": ["target_item"],
                       "stca_dim": 32, "stca_layers": 2, "stca_num_heads": 2, "stca_expansion_ratio": 2,
                       "fields": [{"name": "item", "kind": "categorical", "embedding_dim": 16,
                                   "encoding": {"type": "identity", "max_id": 500, "share_with": "target_item",
                                                "share_embedding": True}}]}]
    m["tokenization"]["num_feature_tokens"] = 4
    m["model"].update({"token_dim": 64, "hidden_dim": 128, "task_head_hidden_dim": 32})
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences = {"clicks": SequenceSpec(fields={"item": FieldSpec(vocab=500)}, max_len=30, min_len=5)}
    return app_config_from_mapping(m), spec


def test_stca_rankmixer_trains_on_cpu():
    cfg, spec = _stca_rankmixer()
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    assert "clicks" in model.summaries.mods
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    losses = [float(tr.train_step(batch).loss) for _ in range(6)]
    assert losses[-1] < losses[0]
    tr.forward_backward(batch)
    name = "summaries.mods.clicks.encoder.layers.1.wk"
    o, n = tr.dense.offsets[name], tr.dense.params[name].numel()
    assert float(tr.dense.grad[o:o + n].abs().sum()) > 0  # the summary reaches the loss


@pytest.mark.gpu
def test_stca_rankmixer_cuda_matches_cpu():
    test_cuda_step_matches_cpu_reference(_stca_rankmixer)
