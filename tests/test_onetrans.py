"""OneTrans model: pyramid schedule, CPU training, CUDA path against the fp32 CPU definition."""

import pytest
import torch

from mdl_b200.config.loader import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config
from mdl_b200.data.synthetic import SyntheticGenerator
from mdl_b200.models.factory import build_model
from mdl_b200.models.onetrans import pyramid_query_counts
from mdl_b200.ops._ext import check_error_word
from mdl_b200.train.trainer import Trainer


def _small(seq_len=40, layers=3, min_len=10, heads=2, schedule="halve", readout="default"):
    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=seq_len, num_layers=layers,
                            pyramid_schedule=schedule)
    m["model"].update({"hidden_dim": 128, "token_dim": 32 * heads, "num_heads": heads, "num_ns_tokens": 4,
                       "task_head_hidden_dim": 64, "pyramid_round_to": 8, "readout": readout})
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences["behavior"].min_len = min_len
    return app_config_from_mapping(m), spec


def test_pyramid_schedules():
    cfg4, _ = scaled_config(4, 1e-3, num_fields=8, batch=8)
    cfg = app_config_from_mapping(cfg4)
    assert pyramid_query_counts(cfg, 512, 32) == [512, 256, 256, 128, 128, 64]
    m, _ = scaled_config(4, 1e-3, num_fields=8, batch=8, pyramid_schedule="linear")
    m["model"]["final_s_tokens"] = 12
    cfg = app_config_from_mapping(m)
    # the reference's linear schedule (src/model.py:6181-6198), rounded to 32
    assert pyramid_query_counts(cfg, 512, 32) == [416, 352, 256, 192, 96, 12]


def test_onetrans_cpu_trains():
    cfg, spec = _small()
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    gen = SyntheticGenerator(model.encoder.batch_plan, spec)
    batch = gen.batch(64)
    losses = [float(tr.train_step(batch).loss) for _ in range(8)]
    assert losses[-1] < losses[0]


def test_onetrans_reference_state_dict_names():
    cfg, _ = _small()
    model = build_model(cfg, device="cpu", base_seed=1)
    sd = model.reference_state_dict()
    assert "backbone.blocks.0.attention.ns_query.3.weight" in sd
    assert sd["backbone.blocks.0.attention.s_key.weight"].shape == (64, 64)
    assert "backbone.tokenizer.auto_ns_projection.2.bias" in sd


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [dict(), dict(seq_len=300, layers=4, min_len=50, heads=4),
                                     dict(readout="task_query")])
def test_onetrans_cuda_step_matches_cpu_reference(variant):
    cfg, spec = _small(**variant)
    torch.manual_seed(0)
    cpu_model = build_model(cfg, device="cpu", base_seed=1)
    gpu_model = build_model(cfg, device="cuda", base_seed=1)
    gpu_model.load_state_dict({k: v.cuda() for k, v in cpu_model.state_dict().items()})
    gpu_model.store.slab.copy_(cpu_model.store.slab)
    cpu_tr = Trainer(cfg, cpu_model, device=torch.device("cpu"))
    gpu_tr = Trainer(cfg, gpu_model, device=torch.device("cuda"))
    gen = SyntheticGenerator(cpu_model.encoder.batch_plan, spec)
    batch = gen.batch(64)
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
        err = ((ref - got).norm() / (ref.norm() + 1e-9)).item()
        assert err < 0.06, f"{name}: grad error {err:.3f}"
    ref = cpu_model.store.grad
    got = gpu_model.store.grad.cpu()
    assert ((ref - got).norm() / (ref.norm() + 1e-9)) < 0.06


# ----------------------------------------------------------------------------- MDL on OneTrans
def _small_mdl(first_seq=None, **model):
    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=3, mdl=True)
    m["model"].update({"hidden_dim": 128, "token_dim": 64, "num_heads": 2, "num_ns_tokens": 4,
                       "task_head_hidden_dim": 64, "pyramid_round_to": 8, "first_domain_sequence_layer": first_seq})
    m["model"].update(model)
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences["behavior"].min_len = 10
    return app_config_from_mapping(m), spec


@pytest.mark.parametrize("variant", [
    dict(),
    dict(first_seq=1),
    dict(mdl_token_state="split"),
    dict(scene_feature_bias="film"),
    dict(use_task_tokens=False),
    dict(use_scenario_tokens=False),
    dict(use_task_feature_interaction=False, use_scenario_feature_interaction=False),
])
def test_mdl_onetrans_cpu_trains(variant):
    cfg, spec = _small_mdl(**variant)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    assert type(model).__name__ == "MDLOneTransModel"
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    out = tr.forward_backward(batch)
    assert out["logits"].shape == (64, 3)
    losses = [float(tr.train_step(batch).loss) for _ in range(8)]
    assert losses[-1] < losses[0]


def test_mdl_onetrans_block_layout():
    cfg, _ = _small_mdl(first_seq=2)
    model = build_model(cfg, device="cpu", base_seed=1)
    assert model.Ns == 6 and model.Nt == 3
    assert [b.scenario_sequence_attention is not None for b in model.blocks] == [False, False, True]
    assert model.blocks[0].task_attention.key_projection.num_tokens == model.num_ns
    # the fixed-width NS readers are not built where the sequence reader replaces them
    assert model.blocks[2].scenario_attention is None
    buckets = model.dense_buckets()
    assert any(n.startswith("blocks.2.") for n in buckets[1]) and any(n.startswith("layers.2.") for n in buckets[1])
    assert sorted(n for g in buckets for n in g) == sorted(n for n, _ in model.named_parameters())


def test_sequence_domain_attention_masks_padding():
    """Keys before ``kstart`` do not change the output (reference
    ``VariableLengthDomainAttention`` masks padded sequence positions)."""

    from mdl_b200.models.mdl import SequenceDomainAttention

    torch.manual_seed(0)
    att = SequenceDomainAttention(32, 4)
    q = torch.randn(3, 5, 32)
    mem = torch.randn(3, 9, 32)
    ks = torch.tensor([0, 3, 8])
    out = att(q, mem, ks)
    mem2 = mem.clone()
    mem2[1, :3] = 100.0
    mem2[2, :8] = -7.0
    torch.testing.assert_close(att(q, mem2, ks), out)
    ref = att(q[2:], mem[2:, 8:], torch.zeros(1, dtype=torch.long))
    torch.testing.assert_close(out[2:], ref)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [dict(), dict(first_seq=1, scene_feature_bias="film")])
def test_mdl_onetrans_cuda_step_matches_cpu_reference(variant):
    cfg, spec = _small_mdl(**variant)
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
        n = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + n], gg[o:o + n]
        err = (ref - got).norm().item()
        assert err <= 0.1 * ref.norm().item() + 2e-3 * scale, (name, err, ref.norm().item())


# ----------------------------------------------------------------------------- NS tokenizers
def _ns_variant(mode, mdl=False, **model):
    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=2, mdl=mdl)
    m["model"].update({"hidden_dim": 128, "token_dim": 64, "num_heads": 2, "num_ns_tokens": 4,
                       "task_head_hidden_dim": 64, "pyramid_round_to": 8, "ns_tokenizer": mode})
    m["model"].update(model)
    if mode == "groupwise":
        feats = [f["name"] for f in m["features"] if f.get("embedding_scope", "feature") == "feature"]
        m["tokenization"]["ns_tokens"] = [{"name": f"g{i}", "inputs": feats[i::3]} for i in range(3)]
    m["training"].update({"lr_warmup_steps": 0, "dense_optimizer": "adam", "lr_dense": 1e-3})
    spec.sequences["behavior"].min_len = 10
    return app_config_from_mapping(m), spec


@pytest.mark.parametrize("mode,mdl,extra", [("dcnv2", False, {}), ("dcnv2", False, {"ns_dcn_low_rank": 16,
                                                                                     "ns_dcn_deep_layers": 0}),
                                            ("groupwise", False, {}), ("groupwise", True, {})])
def test_ns_tokenizers_train(mode, mdl, extra):
    cfg, spec = _ns_variant(mode, mdl, **extra)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    if mode == "groupwise":
        assert model.num_ns == 3
        assert model.encoder.plan.out_width == 0     # the NS inputs come from the per-group plan only
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    losses = [float(tr.train_step(batch).loss) for _ in range(8)]
    assert losses[-1] < losses[0]
    sd = model.reference_state_dict() if not mdl else {}
    if mode == "dcnv2" and not extra:
        assert "backbone.tokenizer.dcn_ns_encoder.cross_layers.2.weight" in sd
        assert sd["backbone.tokenizer.dcn_ns_encoder.output_proj.weight"].shape == (4 * 64, 256)
    if mode == "groupwise" and not mdl:
        assert "backbone.tokenizer.ns_projectors.2.2.bias" in sd


@pytest.mark.gpu
@pytest.mark.parametrize("mode,mdl", [("dcnv2", False), ("groupwise", True)])
def test_ns_tokenizers_cuda_match_cpu(mode, mdl):
    cfg, spec = _ns_variant(mode, mdl)
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
        n = cpu_tr.dense.params[name].numel()
        ref, got = gc[o:o + n], gg[o:o + n]
        err = (ref - got).norm().item()
        assert err <= 0.1 * ref.norm().item() + 2e-3 * scale, (name, err, ref.norm().item())


def test_task_query_readout_trains():
    cfg, spec = _small(layers=2, readout="task_query")
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    assert model.task_query is not None and model.heads_mod.input_dim == 64
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    losses = [float(tr.train_step(batch).loss) for _ in range(8)]
    assert losses[-1] < losses[0]
    assert "task_query_readout.queries" in model.reference_state_dict()
    m, _ = scaled_config(2, 1e-4, num_fields=12, batch=64)
    m["model"]["readout"] = "task_query"
    with pytest.raises(Exception, match="task_query"):
        app_config_from_mapping(m)


# ----------------------------------------------------------------------------- request-level batching
@pytest.mark.parametrize("make", ["onetrans", "longer", "mixformer"])
def test_request_level_sequences_match_expanded_rows(make):
    """Sequences stored once per request (``row_indices``) give the same loss and
    gradients as the same sequences repeated on every candidate row."""

    import copy

    from mdl_b200.data.batch import PackedBatch

    if make == "onetrans":
        cfg, spec = _small(layers=2)
    elif make == "longer":
        from tests.test_longer_mixformer import _longer

        cfg, spec = _longer("mixformer")
    else:
        from tests.test_longer_mixformer import _mixformer

        cfg, spec = _mixformer()
    spec = copy.deepcopy(spec)
    spec.sequences["behavior"].candidates_per_request = 4
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    tr = Trainer(cfg, model, device=torch.device("cpu"))
    b = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    seq = b.sequences["behavior"]
    assert seq["lengths"].numel() == 16 and seq["row_indices"].numel() == 64
    ri = seq["row_indices"]
    L = cfg.sequences[0].max_length
    ids = seq["ids"].view(seq["ids"].shape[0], 16, L)[:, ri].reshape(seq["ids"].shape[0], 64 * L)
    flat = {"ids": ids.clone(), "lengths": seq["lengths"][ri].clone()}
    expanded = PackedBatch.pack(b.ids, b.offsets, b.dense, b.labels, b.label_mask, b.scenario_id, b.rows,
                                sequences={"behavior": flat})
    out_r = tr.forward_backward(b)
    g_r = tr.dense.grad.clone()
    e_r = model.store.grad.clone()
    tr.dense.grad.zero_()
    model.store.grad.zero_()
    out_e = tr.forward_backward(expanded)
    torch.testing.assert_close(out_r["loss"], out_e["loss"])
    torch.testing.assert_close(g_r, tr.dense.grad, atol=1e-6, rtol=1e-4)
    torch.testing.assert_close(e_r, model.store.grad, atol=1e-6, rtol=1e-4)


@pytest.mark.parametrize("dedup", [False, True])
def test_sequence_parquet_round_trip(tmp_path, dedup):
    """Synthetic batch -> Parquet list columns -> tensorizer gives the same sequence payload
    (and, with request deduplication, the same request rows and ``row_indices``)."""

    import copy

    import pyarrow as pa
    import pyarrow.parquet as pq

    from mdl_b200.data.parquet import Tensorizer, write_synthetic_parquet

    m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=2)
    m["model"].update({"hidden_dim": 128, "token_dim": 64, "num_heads": 2, "num_ns_tokens": 4,
                       "task_head_hidden_dim": 64, "pyramid_round_to": 8})
    if dedup:
        m.setdefault("data", {}).setdefault("train", {})["request_id"] = "req"
        m["data"]["train"].setdefault("reader", {})["deduplicate_request_features"] = True
    cfg = app_config_from_mapping(m)
    spec = copy.deepcopy(spec)
    spec.sequences["behavior"].min_len = 5
    spec.sequences["behavior"].candidates_per_request = 4
    model = build_model(cfg, device="cpu", base_seed=1)
    b = SyntheticGenerator(model.encoder.batch_plan, spec).batch(64)
    path = tmp_path / "s.parquet"
    write_synthetic_parquet(str(path), b, model.encoder.batch_plan, cfg)
    t = pq.read_table(path)
    t = t.append_column("req", pa.array(b.sequences["behavior"]["row_indices"].numpy() * 7 + 3))
    tz = Tensorizer(cfg, model.encoder.batch_plan, seq_names=["behavior"])
    got = tz(t).sequences["behavior"]
    want = b.sequences["behavior"]
    if dedup:
        assert torch.equal(got["row_indices"], want["row_indices"])
        assert torch.equal(got["ids"], want["ids"]) and torch.equal(got["lengths"], want["lengths"])
    else:
        ri = want["row_indices"]
        F = want["ids"].shape[0]
        L = 40
        exp = want["ids"].view(F, -1, L)[:, ri].reshape(F, -1)
        assert torch.equal(got["ids"], exp) and torch.equal(got["lengths"], want["lengths"][ri])


@pytest.mark.parametrize("trunc,order,expect", [
    ("tail", "oldest_to_newest", [[0, 0, 1, 2], [3, 4, 5, 6]]),
    ("head", "oldest_to_newest", [[0, 0, 1, 2], [1, 2, 3, 4]]),
    ("tail", "newest_to_oldest", [[0, 0, 2, 1], [6, 5, 4, 3]]),
])
def test_sequence_truncation_layout(trunc, order, expect):
    import pyarrow as pa

    from mdl_b200.data.parquet import Tensorizer

    m, _ = scaled_config(4, 1e-4, num_fields=12, batch=8, seq_len=4, num_layers=1)
    m["sequences"][0].update({"truncation": trunc, "sequence_order": order})
    m["sequences"][0]["fields"] = m["sequences"][0]["fields"][:1]
    cfg = app_config_from_mapping(m)
    tz = Tensorizer(cfg, build_model(cfg, device="cpu", base_seed=1).encoder.batch_plan, seq_names=["behavior"])
    col = pa.array([[1, 2], [1, 2, 3, 4, 5, 6]], type=pa.list_(pa.int64()))
    pos, keep = tz._event_matrix(cfg.sequences[0], col, 2)
    flat = col.values.to_numpy()
    got = [[int(flat[p]) if p >= 0 else 0 for p in row] for row in pos]
    assert got == expect and keep.tolist() == [2, 4]


@pytest.mark.parametrize("ns_mode", ["auto_split", "dcnv2"])
def test_request_cache_matches_full_forward(ns_mode):
    """NS tokens scored against a request cache of the S-token keys give the full
    forward's logits (pyramid layers, padded sequences, requests shared by candidates)."""

    from dataclasses import replace

    cfg, spec = _small(seq_len=40, layers=3, min_len=3)
    if ns_mode != "auto_split":
        m, spec = scaled_config(4, 1e-4, num_fields=12, batch=64, seq_len=40, num_layers=3, pyramid_schedule="halve")
        m["model"].update({"hidden_dim": 128, "token_dim": 64, "num_heads": 2, "num_ns_tokens": 4,
                           "task_head_hidden_dim": 64, "pyramid_round_to": 8, "ns_tokenizer": ns_mode})
        spec.sequences["behavior"].min_len = 3
        cfg = app_config_from_mapping(m)
    torch.manual_seed(0)
    model = build_model(cfg, device="cpu", base_seed=1)
    model.eval()
    batch = SyntheticGenerator(model.encoder.batch_plan, spec).batch(24)
    seq = batch.sequences["behavior"]
    L = cfg.sequences[0].max_length
    nf = seq["ids"].shape[0]
    req = {"ids": seq["ids"].view(nf, 24, L)[:, ::6].reshape(nf, 4 * L), "lengths": seq["lengths"][::6].clone(),
           "row_indices": torch.arange(24) // 6}
    rb = replace(batch, sequences={**batch.sequences, "behavior": req})
    with torch.no_grad():
        full = model(rb)["logits"].float()
        cache = model.precompute_request_cache(rb)
        cached = model.forward_with_cache(rb, cache)
    assert len(cache["layers"]) == 3 and cache["layers"][0][0].shape[0] == 4
    torch.testing.assert_close(cached, full, atol=1e-4, rtol=1e-4)
