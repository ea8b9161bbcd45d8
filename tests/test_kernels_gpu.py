"""GPU numerics of the embedding, norm, head and optimizer kernels vs PyTorch fp32 references."""

import copy

import pytest
import torch
import torch.nn.functional as F

from mdl_b200.ops import embedding as E
from mdl_b200.ops._ext import check_error_word, ext
from mdl_b200.parallel.sharding import EmbeddingTableSpec, plan_embedding_shards

pytestmark = pytest.mark.gpu


def _store_and_plan(device, slice_k=0, slice_stride=0):
    tables = [("ta", 1000, 16), ("tb", 50, 24), ("tc", 3000, 64)]
    plan = plan_embedding_shards([EmbeddingTableSpec(n, r, d) for n, r, d in tables], world_size=1)
    store = E.EmbeddingStore(tables, plan, rank=0, world=1, device=device, init_std=0.1, lr=0.05,
                             initial_accumulator_value=0.1, base_seed=0)
    feats = [
        E.LookupFeature("a", "ta", pooling=E.POOL_NONE, width=16, out_col=0),
        E.LookupFeature("b", "tb", pooling=E.POOL_MEAN, width=24, out_col=16),
        E.LookupFeature("d", None, width=8, out_col=40, dense_col=0),
        E.LookupFeature("c", "tc", pooling=E.POOL_SUM, width=64, out_col=48),
        E.LookupFeature("c2", "tc", pooling=E.POOL_MEAN, width=64, out_col=112),
    ]
    lplan = E.LookupPlan(feats, out_width=176, slice_k=slice_k, slice_stride=slice_stride, dense_width=8)
    return store, lplan


def _batch(rows, plan, seed=0):
    g = torch.Generator().manual_seed(seed)
    ids, lengths = [], []
    vocab = {"a": 1000, "b": 50, "c": 3000, "c2": 3000}
    for f in plan.features:
        if f.table is None:
            lengths.append(torch.zeros(rows, dtype=torch.long))
            continue
        ln = torch.randint(0, 6, (rows,), generator=g) if f.pooling != E.POOL_NONE else torch.ones(rows, dtype=torch.long)
        n = int(ln.sum())
        v = torch.randint(0, vocab[f.name], (n,), generator=g)  # includes padding id 0
        ids.append(v)
        lengths.append(ln)
    offsets = torch.zeros(len(plan.features) * rows + 1, dtype=torch.long)
    offsets[1:] = torch.cumsum(torch.cat(lengths), 0)
    dense = torch.randn(rows, 8, generator=g)
    return torch.cat(ids), offsets, dense


@pytest.mark.parametrize("sliced", [False, True])
def test_embedding_forward_backward_adagrad(sliced):
    rows = 300
    kw = dict(slice_k=44, slice_stride=48) if sliced else {}
    cpu_store, plan = _store_and_plan("cpu", **kw)
    gpu_store, gplan = _store_and_plan("cuda", **kw)
    gpu_store.slab.copy_(cpu_store.slab)
    ids, offsets, dense = _batch(rows, plan)
    ref = E.lookup_reference(cpu_store, plan, ids, offsets, dense, rows)
    anchor = torch.zeros(0, device="cuda", requires_grad=True)
    out = E.fused_lookup(gpu_store, gplan, ids.cuda(), offsets.cuda(), dense.cuda(), rows, anchor)
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=1e-2)
    # backward: push gradients, compare the gradient slabs
    gout = torch.randn(rows, plan.out_ld)
    E.backward_reference(cpu_store, plan, ids, offsets, gout.bfloat16().float(), rows)
    out.backward(gout.cuda().bfloat16())
    torch.cuda.synchronize()
    torch.testing.assert_close(gpu_store.grad.cpu(), cpu_store.grad, atol=2e-3, rtol=1e-3)
    n_touched = int((gpu_store.flags != 0).sum())
    assert n_touched == int(cpu_store._cpu_touched.sum())
    # row-wise Adagrad on the touched rows
    cpu_store.step(lr=0.05)
    gpu_store.step(lr=0.05)
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(gpu_store.slab.cpu(), cpu_store.slab, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(gpu_store.acc.cpu(), cpu_store.acc, atol=1e-6, rtol=1e-4)
    assert float(gpu_store.grad.abs().sum()) == 0.0
    assert int(gpu_store.flags.sum()) == 0


@pytest.mark.parametrize("mix", [True, False])
@pytest.mark.parametrize("B,T,D", [(64, 16, 768), (33, 8, 64), (17, 4, 256)])
def test_layernorm_fused(mix, B, T, D):
    torch.manual_seed(0)
    x = torch.randn(B, T, D, device="cuda").bfloat16()
    r = torch.randn(B, T, D, device="cuda").bfloat16()
    g = torch.randn(D, device="cuda")
    b = torch.randn(D, device="cuda")
    out = torch.empty_like(x)
    mean = torch.empty(B * T, device="cuda")
    rstd = torch.empty_like(mean)
    C = ext()
    C.ln_fwd(x, None if mix else r, g, b, out, mean, rstd, B, T, D, mix, 1e-5)
    xf = x.float().requires_grad_(True)
    rf = r.float().requires_grad_(True)
    gf = g.clone().requires_grad_(True)
    bf = b.clone().requires_grad_(True)
    dh = D // T
    v = (xf.view(B, T, T, dh).permute(0, 2, 1, 3).reshape(B, T, D) + xf) if mix else xf + rf
    ref = F.layer_norm(v, (D,), gf, bf, 1e-5)
    torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)
    dy = torch.randn(B, T, D, device="cuda").bfloat16()
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dx2 = torch.empty_like(x)
    grid = C.ln_bwd_grid(B)
    partials = torch.empty(grid, 2 * D, device="cuda")
    dg = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    C.ln_bwd(dy, None, 1.0, x, None if mix else r, mean, rstd, g, dx, dx2, partials, dg, db, B, T, D, mix, grid)
    torch.cuda.synchronize()
    torch.testing.assert_close(dx.float(), xf.grad, atol=8e-2, rtol=3e-2)
    if not mix:
        torch.testing.assert_close(dx2.float(), rf.grad, atol=8e-2, rtol=3e-2)
    torch.testing.assert_close(dg, gf.grad, atol=0.5, rtol=2e-2)
    torch.testing.assert_close(db, bf.grad, atol=0.5, rtol=2e-2)
    # a residual gradient added in the same pass: dx + res, dx2 unchanged
    res = torch.randn(B, T, D, device="cuda").bfloat16()
    dxr = torch.empty_like(x)
    dx2r = torch.empty_like(x)
    C.ln_bwd(dy, None, 1.0, x, None if mix else r, mean, rstd, g, dxr, dx2r, partials, dg, db, B, T, D, mix, grid,
             res)
    torch.cuda.synchronize()
    torch.testing.assert_close(dxr.float(), dx.float() + res.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(dx2r, dx2)


@pytest.mark.parametrize("D", [256, 512, 1024])
def test_rmsnorm(D):
    torch.manual_seed(0)
    R = 300
    x = torch.randn(R, D, device="cuda").bfloat16()
    w = torch.randn(D, device="cuda")
    out = torch.empty_like(x)
    rstd = torch.empty(R, device="cuda")
    C = ext()
    C.rms_fwd(x, w, out, rstd, R, D, 1e-6)
    xf = x.float().requires_grad_(True)
    wf = w.clone().requires_grad_(True)
    ref = xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + 1e-6) * wf
    torch.testing.assert_close(out.float(), ref, atol=5e-2, rtol=2e-2)
    dy = torch.randn(R, D, device="cuda").bfloat16()
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device="cuda")
    C.rms_bwd(x, w, rstd, dy, dx, dw, R, D)
    torch.cuda.synchronize()
    torch.testing.assert_close(dx.float(), xf.grad, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(dw, wf.grad, atol=0.3, rtol=2e-2)


def test_rmsnorm_backward_residual():
    """dx += residual gradient: same layout, and the last `tail` rows of each sample."""

    torch.manual_seed(1)
    Bs, period, tail, D = 7, 50, 20, 256
    R = Bs * period
    x = torch.randn(R, D, device="cuda").bfloat16()
    w = torch.randn(D, device="cuda")
    out, rstd = torch.empty_like(x), torch.empty(R, device="cuda")
    C = ext()
    C.rms_fwd(x, w, out, rstd, R, D, 1e-6)
    dy = torch.randn(R, D, device="cuda").bfloat16()
    base = torch.empty_like(x)
    C.rms_bwd(x, w, rstd, dy, base, None, R, D)
    same = torch.randn(R, D, device="cuda").bfloat16()
    dx = torch.empty_like(x)
    C.rms_bwd(x, w, rstd, dy, dx, None, R, D, dres=same)
    torch.testing.assert_close(dx.float(), base.float() + same.float(), atol=3e-2, rtol=1e-2)
    part = torch.randn(Bs * tail, D, device="cuda").bfloat16()
    C.rms_bwd(x, w, rstd, dy, dx, None, R, D, dres=part, res_period=period, res_tail=tail)
    want = base.float().view(Bs, period, D).clone()
    want[:, period - tail:] += part.float().view(Bs, tail, D)
    torch.testing.assert_close(dx.float(), want.view(R, D), atol=3e-2, rtol=1e-2)


def test_head_bce():
    torch.manual_seed(0)
    B, nt, H = 500, 3, 256
    pre = torch.randn(B, nt * H, device="cuda").bfloat16()
    act = F.gelu(pre.float()).bfloat16()
    w2 = torch.randn(nt, H, device="cuda") * 0.1
    b2 = torch.randn(nt, device="cuda")
    labels = (torch.rand(B, nt, device="cuda") < 0.3).float()
    mask = (torch.rand(B, nt, device="cuda") < 0.9).float()
    scale = torch.tensor([0.5, 1.0, 2.0], device="cuda")
    logits = torch.empty(B, nt, device="cuda")
    loss = torch.zeros(1, device="cuda")
    dpre = torch.empty_like(pre)
    dw2 = torch.zeros_like(w2)
    db2 = torch.zeros_like(b2)
    ext().head_bce(act, pre, w2, b2, labels, mask, scale, logits, loss, dpre, dw2, db2, B, nt, H, False)
    pf = pre.float().requires_grad_(True)
    w2f = w2.clone().requires_grad_(True)
    b2f = b2.clone().requires_grad_(True)
    a = F.gelu(pf).view(B, nt, H)
    z = (a * w2f.unsqueeze(0)).sum(-1) + b2f
    l = (F.binary_cross_entropy_with_logits(z, labels, reduction="none") * mask * scale).sum()
    l.backward()
    torch.cuda.synchronize()
    torch.testing.assert_close(logits, z.detach(), atol=3e-2, rtol=1e-2)
    torch.testing.assert_close(loss[0], l.detach(), atol=0.5, rtol=1e-2)
    torch.testing.assert_close(dpre.float(), pf.grad, atol=2e-3, rtol=3e-2)
    torch.testing.assert_close(dw2, w2f.grad, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(db2, b2f.grad, atol=5e-2, rtol=2e-2)


@pytest.mark.parametrize("opt", ["adam", "rmsprop"])
def test_dense_optimizer(opt):
    from mdl_b200.ops.dense import DenseParams

    torch.manual_seed(0)
    ps = [torch.nn.Parameter(torch.randn(37, 11)), torch.nn.Parameter(torch.randn(100))]
    ps_gpu = [torch.nn.Parameter(p.detach().clone().cuda()) for p in ps]
    a = DenseParams([("w", ps[0]), ("b", ps[1])], device="cpu", optimizer=opt, lr=1e-2)
    b = DenseParams([("w", ps_gpu[0]), ("b", ps_gpu[1])], device="cuda", bf16_names={"w"}, optimizer=opt, lr=1e-2)
    for step in range(3):
        g = torch.randn(a.total)
        a.grad.copy_(g)
        b.grad.copy_(g.cuda())
        a.step(clip_norm=5.0)
        b.step(clip_norm=5.0)
    torch.testing.assert_close(b.master.cpu(), a.master, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(ps_gpu[0]._mdl_shadow.float().cpu(), ps[0].detach(), atol=2e-2, rtol=1e-2)


def _small_rankmixer_config():
    from mdl_b200.config import app_config_from_mapping
    from mdl_b200.data.baseline_configs import scaled_config

    m, spec = scaled_config(2, 0.0005, num_fields=24, batch=256)
    m["model"].update({"token_dim": 256, "hidden_dim": 512, "task_head_hidden_dim": 256})
    m["tokenization"]["num_feature_tokens"] = 8
    return app_config_from_mapping(m), spec


def test_rankmixer_cuda_step_matches_cpu_reference():
    from mdl_b200.data.synthetic import SyntheticGenerator
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    cfg, spec = _small_rankmixer_config()
    torch.manual_seed(0)
    cpu_model = build_model(cfg, device="cpu", base_seed=1)
    torch.manual_seed(0)
    gpu_model = build_model(cfg, device="cuda", base_seed=1)
    gpu_model.load_state_dict({k: v.cuda() for k, v in cpu_model.state_dict().items()})
    gpu_model.store.slab.copy_(cpu_model.store.slab)
    cpu_tr = Trainer(cfg, cpu_model, device=torch.device("cpu"))
    gpu_tr = Trainer(cfg, gpu_model, device=torch.device("cuda"))
    gen = SyntheticGenerator(cpu_model.encoder.batch_plan, spec)
    batch = gen.batch(256)
    out_c = cpu_tr.forward_backward(batch)
    out_g = gpu_tr.forward_backward(batch.to("cuda"))
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(out_g["logits"].cpu(), out_c["logits"].detach(), atol=5e-2, rtol=5e-2)
    torch.testing.assert_close(out_g["loss"].cpu(), out_c["loss"].detach(), atol=2e-2, rtol=2e-2)
    # gradients of every dense parameter (flat buffers share one layout)
    gc, gg = cpu_tr.dense.grad, gpu_tr.dense.grad.cpu()
    for name in cpu_tr.dense.names:
        o = cpu_tr.dense.offsets[name]
        n = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + n], gg[o:o + n]
        scale = ref.abs().max().item() + 1e-6
        err = (ref - got).abs().max().item() / scale
        assert err < 0.08, f"{name}: relative grad error {err:.3f}"
    # embedding gradients
    ref = cpu_model.store.grad
    got = gpu_model.store.grad.cpu()
    assert ((ref - got).abs().max() / (ref.abs().max() + 1e-9)) < 0.08


@pytest.mark.parametrize("rows,frac", [(1000, 0.3), (100003, 0.01), (5_000_017, 0.001)])
def test_compact_touched_lists_every_flagged_row(rows, frac):
    flags = torch.zeros((rows + 511) // 512 * 512, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(0)
    hit = torch.rand(rows, device="cuda", generator=g) < frac
    flags[:rows][hit] = 1
    lst = torch.empty(rows, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ext().compact_touched(flags, rows, lst, cnt)
    torch.cuda.synchronize()
    n = int(cnt.item())
    assert n == int(hit.sum().item())
    got = torch.sort(lst[:n].long()).values
    want = hit.nonzero().flatten()
    assert torch.equal(got, want)
    assert int(flags.sum().item()) == 0
