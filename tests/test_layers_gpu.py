"""GPU numerics of the MDL building blocks (few-query attention, per-token FFN,
Linear, task heads) and of the MDL model vs PyTorch fp32 references."""

import math

import pytest
import torch
import torch.nn.functional as F

from mdl_b200.ops._ext import check_error_word

pytestmark = pytest.mark.gpu


def _register(module, device="cuda"):
    """Put a module's parameters into flat DenseParams storage (bf16 shadows + grad views)."""

    from mdl_b200.ops.dense import DenseParams

    return DenseParams(module.named_parameters(), device=torch.device(device))


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("Nq,Nk,H,hd,masked", [(21, 16, 12, 64, False), (3, 16, 8, 32, False), (7, 40, 4, 128, True),
                                              (64, 64, 2, 16, True)])
def test_few_query_attention_matches_sdpa(Nq, Nk, H, hd, masked):
    from mdl_b200.ops.layers import few_query_attention

    torch.manual_seed(0)
    B, D = 37, H * hd
    q = torch.randn(B, Nq, D, device="cuda").to(torch.bfloat16).requires_grad_(True)
    k = torch.randn(B, Nk, D, device="cuda").to(torch.bfloat16).requires_grad_(True)
    v = torch.randn(B, Nk, D, device="cuda").to(torch.bfloat16).requires_grad_(True)
    kv = torch.randint(1, Nk + 1, (B,), device="cuda") if masked else None
    out = few_query_attention(q, k, v, H, kv)
    dout = torch.randn_like(out)
    out.backward(dout)
    torch.cuda.synchronize()
    check_error_word(0)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    qh = qf.view(B, Nq, H, hd).transpose(1, 2)
    kh = kf.view(B, Nk, H, hd).transpose(1, 2)
    vh = vf.view(B, Nk, H, hd).transpose(1, 2)
    s = qh @ kh.transpose(-1, -2) / math.sqrt(hd)
    if kv is not None:
        s = s.masked_fill(torch.arange(Nk, device="cuda").view(1, 1, 1, Nk) >= kv.view(B, 1, 1, 1), float("-inf"))
    ref = (torch.softmax(s, -1) @ vh).transpose(1, 2).reshape(B, Nq, D)
    ref.backward(dout.float())
    assert _rel(out, ref) < 2e-2
    for got, want in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert _rel(got, want) < 3e-2


@pytest.mark.parametrize("act,out_relu,strided", [("gelu", False, False), ("relu", True, True), ("gelu", True, True)])
def test_per_token_ffn_matches_reference(act, out_relu, strided):
    from mdl_b200.ops.layers import PerTokenFFN

    torch.manual_seed(0)
    N, Din, H, Do, B = 5, 64, 192, 128, 300
    m = PerTokenFFN(N, Din, H, act, output_relu=out_relu, device="cuda", out_dim=Do)
    m.restrict_inputs([40, 64, 8, 56, 64])
    ref_w = {n: p.detach().clone() for n, p in m.named_parameters()}
    dp = _register(m)
    full = torch.randn(B, N + 3, Din, device="cuda")
    for t, w in enumerate([40, 64, 8, 56, 64]):
        full[:, t, w:] = 0
    xin = full.to(torch.bfloat16)
    if strided:
        base = xin.detach().clone().requires_grad_(True)
        x = base[:, :N]
    else:
        x = xin[:, :N].contiguous().requires_grad_(True)
    y = m(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    check_error_word(0)
    xf = x.detach().float().requires_grad_(True)
    wi, bi, wo, bo = (ref_w[k].clone().requires_grad_(True) for k in
                      ("input_weight", "input_bias", "output_weight", "output_bias"))
    actf = F.relu if act == "relu" else F.gelu
    h = actf(torch.einsum("bnd,nhd->bnh", xf, wi.to(torch.bfloat16).float()) + bi)
    yr = torch.einsum("bnh,ndh->bnd", h, wo.to(torch.bfloat16).float()) + bo
    if out_relu:
        # follow the kernel's activation pattern: a pre-activation within bf16 rounding of 0
        # may land on either side, which is not what this test measures
        yr = yr * (y.detach().float() > 0)
    yr.backward(dy.float())
    assert _rel(y, yr) < 2e-2
    g = dict(zip(("input_weight", "input_bias", "output_weight", "output_bias"), (wi, bi, wo, bo)))
    for name, p in g.items():
        got = m.get_parameter(name)._mdl_grad
        assert _rel(got, p.grad) < 3e-2, name
    gx = base.grad[:, :N] if strided else x.grad
    assert _rel(gx, xf.grad) < 3e-2
    if strided:
        assert base.grad[:, N:].abs().max().item() == 0.0
    # zero-padded input columns keep a zero weight gradient
    assert m.input_weight._mdl_grad[2, :, 8:].abs().max().item() == 0.0
    del dp


def test_linear_matches_reference():
    from mdl_b200.ops.layers import Linear

    torch.manual_seed(0)
    m = Linear(256, 1536, device="cuda")
    w0, b0 = m.weight.detach().clone(), m.bias.detach().clone()
    dp = _register(m)
    x = torch.randn(777, 256, device="cuda").to(torch.bfloat16).requires_grad_(True)
    y = m(x)
    dy = torch.randn_like(y)
    y.backward(dy)
    torch.cuda.synchronize()
    check_error_word(0)
    xf = x.detach().float().requires_grad_(True)
    wf = w0.to(torch.bfloat16).float().requires_grad_(True)
    bf = b0.clone().requires_grad_(True)
    yr = xf @ wf.t() + bf
    yr.backward(dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(m.weight._mdl_grad, wf.grad) < 2e-2
    assert _rel(m.bias._mdl_grad, bf.grad) < 2e-2
    assert _rel(x.grad, xf.grad) < 2e-2
    del dp


@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_task_heads_match_reference(act):
    from mdl_b200.models.heads import TaskHeads

    torch.manual_seed(0)
    nt, D, Hh, B = 3, 256, 192, 500
    m = TaskHeads(nt, D, Hh, act, device="cuda")
    ref = {n: p.detach().clone() for n, p in m.named_parameters()}
    dp = _register(m)
    x = torch.randn(B, nt, D, device="cuda").to(torch.bfloat16).requires_grad_(True)
    labels = (torch.rand(B, nt, device="cuda") < 0.3).float()
    mask = (torch.rand(B, nt, device="cuda") < 0.8).float()
    scale = torch.tensor([1.0 / B, 2.0 / B, 0.5 / B], device="cuda")
    out = m(x, labels, mask, scale)
    out["loss"].backward()
    torch.cuda.synchronize()
    check_error_word(0)
    xf = x.detach().float().requires_grad_(True)
    w1 = ref["w1"].to(torch.bfloat16).float().requires_grad_(True)
    b1, w2, b2 = (ref[k].clone().requires_grad_(True) for k in ("b1", "w2", "b2"))
    actf = F.relu if act == "relu" else F.gelu
    hid = actf(torch.einsum("btd,thd->bth", xf, w1) + b1)
    logits = (hid * w2).sum(-1) + b2
    loss = (F.binary_cross_entropy_with_logits(logits, labels, reduction="none") * mask * scale).sum()
    loss.backward()
    assert _rel(out["logits"], logits) < 2e-2
    assert abs(out["loss"].item() - loss.item()) < 2e-2 * abs(loss.item())
    for name, p in (("w1", w1), ("b1", b1), ("w2", w2), ("b2", b2)):
        assert _rel(m.get_parameter(name)._mdl_grad, p.grad) < 4e-2, name
    assert _rel(x.grad, xf.grad) < 4e-2
    del dp


def _small_mdl_config(**model):
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import scaled_config

    m, spec = scaled_config(3, 0.001, num_fields=24, batch=256)
    m["model"].update({"token_dim": 256, "hidden_dim": 512, "task_head_hidden_dim": 256, "num_heads": 4})
    m["model"].update(model)
    m["tokenization"]["num_feature_tokens"] = 8
    return app_config_from_mapping(m), spec


@pytest.mark.parametrize("variant", [{}, {"mdl_token_state": "split", "scene_feature_bias": "none"},
                                     {"mdl_feature_interaction": "direct_ffn", "scene_feature_bias": "additive"}])
def test_mdl_cuda_step_matches_cpu_reference(variant):
    from mdl_b200.data.synthetic import SyntheticGenerator
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    cfg, spec = _small_mdl_config(**variant)
    torch.manual_seed(0)
    cpu_model = build_model(cfg, device="cpu", base_seed=1)
    torch.manual_seed(0)
    gpu_model = build_model(cfg, device="cuda", base_seed=1)
    gpu_model.load_state_dict({k: v.cuda() for k, v in cpu_model.state_dict().items()})
    gpu_model.store.slab.copy_(cpu_model.store.slab)
    if cfg.model.scene_feature_bias != "none":
        # non-zero FiLM weights so the scene path is exercised
        with torch.no_grad():
            w = torch.randn_like(cpu_model.scene_feature_bias.weight) * 0.02
            cpu_model.scene_feature_bias.weight.copy_(w)
            gpu_model.scene_feature_bias.weight.copy_(w.cuda())
    cpu_tr = Trainer(cfg, cpu_model, device=torch.device("cpu"))
    gpu_tr = Trainer(cfg, gpu_model, device=torch.device("cuda"))
    gen = SyntheticGenerator(cpu_model.encoder.batch_plan, spec)
    batch = gen.batch(256)
    out_c = cpu_tr.forward_backward(batch)
    out_g = gpu_tr.forward_backward(batch.to("cuda"))
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(out_g["logits"].cpu(), out_c["logits"].detach(), atol=6e-2, rtol=6e-2)
    torch.testing.assert_close(out_g["loss"].cpu(), out_c["loss"].detach(), atol=3e-2, rtol=3e-2)
    gc, gg = cpu_tr.dense.grad, gpu_tr.dense.grad.cpu()
    for name in cpu_tr.dense.names:
        o = cpu_tr.dense.offsets[name]
        n = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + n], gg[o:o + n]
        # bf16 activations put a few ReLU inputs on the other side of zero: bound the
        # norm-relative error tightly and the worst element loosely
        err = ((ref - got).norm() / (ref.norm() + 1e-9)).item()
        worst = ((ref - got).abs().max() / (ref.abs().max() + 1e-9)).item()
        assert err < 0.05 and worst < 0.2, f"{name}: grad error {err:.3f} (worst {worst:.3f})"
    ref = cpu_model.store.grad
    got = gpu_model.store.grad.cpu()
    assert ((ref - got).norm() / (ref.norm() + 1e-9)) < 0.05
