"""LONGER token merger (``longer_token_merge``) and inner blocks (``longer_inner_layers``):
slot order, padding, identity of zero-parameter inner blocks, inner blocks against a
per-group loop, CPU training, and the CUDA path against the CPU definition."""

import pytest
import torch

from mdl_b200.config.loader import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.ops._ext import check_error_word
from mdl_b200.train.trainer import Trainer


def _cfg(merge=2, inner=0, d=8, heads=2, seq_len=40, R=8, min_len=3):
    m, spec = scaled_config(5, 1e-4, num_fields=12, batch=32, seq_len=seq_len, min_len=min_len, query_tokens=R,
                            self_layers=1, d=d, heads=heads, sequence_head="none", ns_tokens=4)
    m["sequences"][0].update({"longer_token_merge": merge, "longer_inner_layers": inner})
    m["model"].update({"token_dim": 16, "hidden_dim": 64, "task_head_hidden_dim": 32})
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    return app_config_from_mapping(m), spec


def _encoder(**kw):
    cfg, spec = _cfg(**kw)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    return model, model.longer, cfg, spec


def test_merge_concatenates_slots_in_order_and_zeroes_padding():
    _, enc, _, _ = _encoder(merge=2, d=2, heads=1)
    tok = torch.tensor([[[1.0, 2.0], [3.0, 4.0], [5.0, 6.0], [7.0, 8.0], [9.0, 10.0]]])
    merged, kst = enc.merge_tokens(tok, torch.tensor([1], dtype=torch.int32), native=False)
    # L=5 is left-padded to 6; padding events (the pad and the first event) read as zero
    assert merged.shape == (1, 3, 4) and int(kst) == 1
    torch.testing.assert_close(merged, torch.tensor([[[0.0, 0.0, 0.0, 0.0], [3.0, 4.0, 5.0, 6.0],
                                                      [7.0, 8.0, 9.0, 10.0]]]))
    assert enc.D == 4 and enc.Din == 2


def test_zero_parameter_inner_blocks_are_identity():
    _, enc, _, _ = _encoder(merge=2, inner=1, d=4, heads=1)
    for p in enc.inner.parameters():
        torch.nn.init.zeros_(p)
    tok = torch.arange(24, dtype=torch.float32).view(1, 6, 4)
    merged, _ = enc.merge_tokens(tok, torch.tensor([0], dtype=torch.int32), native=False)
    torch.testing.assert_close(merged, tok.view(1, 3, 8))


def test_inner_blocks_match_a_per_group_loop():
    _, enc, _, _ = _encoder(merge=3, inner=2, d=8, heads=2)
    torch.manual_seed(3)
    B, L, Din = 3, 10, 8
    tok = torch.randn(B, L, Din)
    kst = torch.tensor([0, 4, 10], dtype=torch.int32)  # full, partial, empty sequence
    merged, mk = enc.merge_tokens(tok, kst, native=False)
    pad = (-L) % 3
    assert merged.shape == (B, (L + pad) // 3, 24)
    assert mk.tolist() == [(k + pad) // 3 for k in kst.tolist()]
    x = torch.nn.functional.pad(tok, (0, 0, pad, 0))
    for b in range(B):
        k = int(kst[b]) + pad
        for g in range((L + pad) // 3):
            grp = x[b:b + 1, 3 * g:3 * g + 3]
            gk = torch.tensor([min(max(k - 3 * g, 0), 3)], dtype=torch.int32)
            h = grp
            for blk in enc.inner:
                h = blk.forward_reference(h, gk, 3, enc.heads, False, 0)
            slot_valid = (torch.arange(3) + 3 * g >= k).float().view(1, 3, 1)
            want = (h * slot_valid).reshape(24)
            torch.testing.assert_close(merged[b, g], want, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("merge,inner", [(2, 0), (4, 1)])
def test_merged_longer_trains_on_cpu(merge, inner):
    model, enc, cfg, spec = _encoder(merge=merge, inner=inner, d=8, heads=2)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(32)
    losses = [float(tr.train_step(batch).loss) for _ in range(6)]
    assert losses[-1] < losses[0]
    assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())


@pytest.mark.gpu
@pytest.mark.parametrize("merge,inner,d,heads", [
    (2, 0, 16, 1),   # merged blocks at head_dim 32: tcgen05 flash attention
    (1, 0, 32, 4),   # the reference's production LONGER widths (head_dim 8): CUDA-core attention
    (2, 1, 32, 4),   # inner blocks at head_dim 8, merged blocks at 16
])
def test_merged_longer_cuda_matches_cpu(merge, inner, d, heads):
    cfg, spec = _cfg(merge=merge, inner=inner, d=d, heads=heads, seq_len=120, R=24, min_len=20)
    torch.manual_seed(0)
    cpu_model = build_model(cfg, device="cpu", base_seed=1)
    gpu_model = build_model(cfg, device="cuda", base_seed=1)
    gpu_model.load_state_dict({k: v.cuda() for k, v in cpu_model.state_dict().items()})
    gpu_model.store.slab.copy_(cpu_model.store.slab)
    cpu_tr = Trainer(cfg, cpu_model, device=torch.device("cpu"))
    gpu_tr = Trainer(cfg, gpu_model, device=torch.device("cuda"))
    batch = SyntheticGenerator(cpu_model.encoder.batch_plan, spec).batch(32)
    out_c = cpu_tr.forward_backward(batch)
    out_g = gpu_tr.forward_backward(batch.to("cuda"))
    torch.cuda.synchronize()
    check_error_word(0)
    torch.testing.assert_close(out_g["logits"].cpu(), out_c["logits"].detach(), atol=6e-2, rtol=6e-2)
    gc, gg = cpu_tr.dense.grad, gpu_tr.dense.grad.cpu()
    assert ((gc - gg).norm() / gc.norm()) < 0.08


def test_request_side_outputs_do_not_depend_on_the_candidate():
    """Candidate global tokens are seen by no other token: changing the candidate's
    inputs changes only the candidate outputs (what makes the request side cacheable)."""

    m, spec = scaled_config(5, 1e-4, num_fields=12, batch=16, seq_len=40, min_len=5, query_tokens=6,
                            self_layers=2, d=16, heads=2, sequence_head="none", ns_tokens=4)
    m["sequences"][0].update({"longer_candidate_global_tokens": 2})
    m["model"].update({"token_dim": 16, "hidden_dim": 64, "task_head_hidden_dim": 32})
    cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    enc = model.longer
    assert enc.Gc == 2
    B, L = 4, enc.L
    torch.manual_seed(5)
    tokens = torch.randn(B, L, enc.Din)
    lengths = torch.tensor([40, 17, 3, 0])
    k_in = enc.cand_mlp.k_in
    t1, t2 = torch.randn(B, k_in), torch.randn(B, k_in)
    u = torch.randn(B, enc.user_mlp.k_in) if enc.Gu else None
    x1 = enc(None, lengths, t1, u, False, tokens=tokens)
    x2 = enc(None, lengths, t2, u, False, tokens=tokens)
    n_req = enc.R + enc.Gu + enc.Gx
    torch.testing.assert_close(x1[:, :n_req], x2[:, :n_req])
    assert (x1[:, n_req:] - x2[:, n_req:]).abs().max() > 1e-3


@pytest.mark.parametrize("merge,inner,cand", [(1, 0, 1), (2, 1, 2)])
def test_request_cache_matches_full_forward(merge, inner, cand):
    """Scoring candidates from a request cache gives the full forward's logits: requests
    shared by several candidates (request-level batching), candidate features per row."""

    m, spec = scaled_config(5, 1e-4, num_fields=12, batch=24, seq_len=40, min_len=5, query_tokens=6,
                            self_layers=2, d=8, heads=2, sequence_head="none", ns_tokens=4)
    m["sequences"][0].update({"longer_candidate_global_tokens": cand, "longer_token_merge": merge,
                              "longer_inner_layers": inner})
    m["model"].update({"token_dim": 16, "hidden_dim": 64, "task_head_hidden_dim": 32})
    cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    model.eval()
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(24)
    seq = batch.sequences["behavior"]
    # three requests of eight candidates each: candidates share their request's events
    ri = torch.arange(24) // 8
    L = cfg.sequences[0].max_length
    ids = seq["ids"].view(seq["ids"].shape[0], 24, L)[:, ::8].reshape(seq["ids"].shape[0], 3 * L)
    req = {"ids": ids, "lengths": seq["lengths"][::8].clone(), "row_indices": ri}
    from dataclasses import replace

    rb = replace(batch, sequences={**batch.sequences, "behavior": req})
    with torch.no_grad():
        full = model(rb)["logits"]
        cache = model.precompute_request_cache(rb)
        assert cache["out"].shape[0] == 3
        cached = model.forward_with_cache(rb, cache)
    torch.testing.assert_close(cached, full.float(), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("self_layers", [0, 2])
def test_summary_only_equals_the_global_slice(self_layers):
    """``summary_only`` computes only the global queries in the last block: the same global
    tokens as the full forward."""

    m, spec = scaled_config(5, 1e-4, num_fields=12, batch=8, seq_len=30, min_len=3, query_tokens=6,
                            self_layers=self_layers, d=16, heads=2, sequence_head="none", ns_tokens=4)
    m["sequences"][0].update({"longer_candidate_global_tokens": 2})
    cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    enc = build_model(cfg, device="cpu", base_seed=1).longer
    torch.manual_seed(2)
    B = 5
    tokens = torch.randn(B, enc.L, enc.Din)
    lengths = torch.tensor([30, 11, 3, 1, 0])
    t_in = torch.randn(B, enc.cand_mlp.k_in)
    u_in = torch.randn(B, enc.user_mlp.k_in) if enc.Gu else None
    with torch.no_grad():
        full = enc(None, lengths, t_in, u_in, False, tokens=tokens)
        summ = enc(None, lengths, t_in, u_in, False, tokens=tokens, summary_only=True)
    assert summ.shape[1] == enc.G
    torch.testing.assert_close(summ, full[:, full.shape[1] - enc.G:], atol=1e-5, rtol=1e-5)
