"""GPU numerics of the sequence paths that feed tokens: sequence summaries
(``mean_pool``, ``attention_pool``, ``longer``) in a ``groupwise`` RankMixer, and
several raw sequences fused into OneTrans S tokens (``intent_ordered`` with SEP
tokens) and MixFormer behaviour tokens (``timestamp_aware``). The native
(bf16, sm_100a kernels) forward and backward are compared with the fp32 PyTorch
definition of the same model (``runtime.kernel_backend: torch``, same seeds)."""

import copy

import pytest
import torch

from mdl_b200.config import app_config_from_mapping
from mdl_b200.data.baseline_configs import scaled_config

pytestmark = pytest.mark.gpu


def _seq(name, L, encoder, **extra):
    fields = [{"name": "item", "kind": "categorical", "source": f"{name}_item", "embedding_dim": 16,
               "encoding": {"type": "identity", "max_id": 5000}},
              {"name": "cat", "kind": "categorical", "source": f"{name}_cat", "embedding_dim": 8,
               "encoding": {"type": "identity", "max_id": 300}},
              {"name": "age", "kind": "dense", "source": f"{name}_age", "dimension": 1}]
    return {"name": name, "fields": fields, "max_length": L, "encoder": encoder, "sequence_order": "oldest_to_newest",
            "truncation": "tail", "time_delta_field": "age", **extra}


def _base(name, batch=96):
    m, _spec = scaled_config(2, 0.0005, num_fields=16, batch=batch)
    m["model"]["name"] = name
    return m


def _rankmixer_mapping():
    m = _base("rankmixer")
    feats = [f["name"] for f in m["features"]]
    m["sequences"] = [
        _seq("hist_mean", 24, "mean_pool", pool_dim=32),
        _seq("hist_att", 24, "attention_pool", pool_dim=32, target_inputs=[feats[0], feats[1]]),
        _seq("hist_longer", 40, "longer", longer_dim=32, longer_num_heads=1, longer_query_tokens=8,
             longer_self_layers=1, longer_cls_tokens=1, longer_user_global_tokens=1,
             longer_user_global_inputs=[feats[2]], longer_candidate_global_tokens=1, rankmixer_summary_tokens=3,
             target_inputs=[feats[0]], longer_output="summary"),
    ]
    groups = [{"name": f"g{i}", "inputs": feats[i * 4:(i + 1) * 4]} for i in range(4)]
    groups += [{"name": "s_mean", "inputs": ["hist_mean"]}, {"name": "s_att", "inputs": ["hist_att"]},
               {"name": "s_longer", "inputs": ["hist_longer"]}, {"name": "dense", "inputs": [feats[-1]]}]
    m["tokenization"] = {"feature_tokenizer": "groupwise", "feature_tokens": groups}
    m["model"].update({"token_dim": 256, "hidden_dim": 512, "task_head_hidden_dim": 128, "num_heads": 8})
    return m


def _stca_rankmixer_mapping():
    """STCA summaries (native path: the shared-history single-query attention kernels) with
    2 heads of width 128 and 4 heads of width 64 over 256-wide histories."""

    m = _base("rankmixer")
    feats = [f["name"] for f in m["features"]]
    m["sequences"] = [
        _seq("hist_stca", 30, "stca", stca_dim=256, stca_layers=2, stca_num_heads=2, stca_expansion_ratio=2,
             target_inputs=[feats[0], feats[1]]),
        _seq("hist_stca4", 20, "stca", stca_dim=256, stca_layers=1, stca_num_heads=4, stca_expansion_ratio=2,
             target_inputs=[feats[2]]),
    ]
    groups = [{"name": f"g{i}", "inputs": feats[i * 3:(i + 1) * 3]} for i in range(5)]
    groups += [{"name": "s_stca", "inputs": ["hist_stca"]}, {"name": "s_stca4", "inputs": ["hist_stca4"]},
               {"name": "dense", "inputs": [feats[-1]]}]
    m["tokenization"] = {"feature_tokenizer": "groupwise", "feature_tokens": groups}
    m["model"].update({"token_dim": 256, "hidden_dim": 512, "task_head_hidden_dim": 128, "num_heads": 8})
    return m


def _onetrans_mapping():
    m = _base("onetrans")
    m["sequences"] = [_seq("s_a", 48, "raw"), _seq("s_b", 32, "raw"), _seq("s_c", 24, "raw")]
    m["tokenization"] = {"feature_tokenizer": "auto_split", "num_feature_tokens": 8,
                         "sequence_tokens": [{"name": n, "inputs": [n]} for n in ("s_a", "s_b", "s_c")]}
    m["model"].update({"token_dim": 64, "num_heads": 2, "hidden_dim": 256, "task_head_hidden_dim": 128,
                       "num_layers": 2, "ns_tokenizer": "auto_split", "num_ns_tokens": 8, "use_sep_tokens": True,
                       "sequence_fusion": "intent_ordered", "use_pyramid": False})
    return m


def _mixformer_mapping():
    m = _base("mixformer")
    m["sequences"] = [_seq("s_a", 40, "raw"), _seq("s_b", 24, "raw")]
    m["tokenization"] = {"feature_tokenizer": "rankmixer", "num_feature_tokens": 4,
                         "sequence_tokens": [{"name": n, "inputs": [n]} for n in ("s_a", "s_b")]}
    m["model"].update({"token_dim": 64, "num_heads": 2, "hidden_dim": 256, "task_head_hidden_dim": 128,
                       "num_layers": 2, "num_ns_tokens": 4, "sequence_fusion": "timestamp_aware",
                       "global_sequence_max_length": 48, "use_sep_tokens": False})
    return m


def _build(mapping, backend):
    from mdl_b200.data.synthetic import SyntheticGenerator, synthetic_spec_from_config
    from mdl_b200.models.factory import build_model
    from mdl_b200.train.trainer import Trainer

    mp = copy.deepcopy(mapping)
    mp["runtime"]["kernel_backend"] = backend
    cfg = app_config_from_mapping(mp)
    torch.manual_seed(0)
    model = build_model(cfg, device=torch.device("cuda", 0), base_seed=0)
    trainer = Trainer(cfg, model, device=torch.device("cuda", 0))
    enc = model.encoder
    seqs = [s for s in cfg.sequences if s.name in enc.seq_plans]
    spec = synthetic_spec_from_config(cfg, enc.batch_plan, sequences=seqs, seed=3)
    batch = SyntheticGenerator(enc.batch_plan, spec).batch(96).to(torch.device("cuda", 0))
    return model, trainer, batch


@pytest.mark.parametrize("make", [_rankmixer_mapping, _stca_rankmixer_mapping, _onetrans_mapping,
                                  _mixformer_mapping])
def test_native_matches_fp32_definition(make):
    from mdl_b200.ops._ext import check_error_word

    mapping = make()
    m_nat, t_nat, batch = _build(mapping, "native")
    m_ref, t_ref, batch_ref = _build(mapping, "torch")
    out_nat = t_nat.forward_backward(batch)
    out_ref = t_ref.forward_backward(batch_ref)
    torch.cuda.synchronize()
    check_error_word(0)
    ln, lr = float(out_nat["loss"]), float(out_ref["loss"])
    assert abs(ln - lr) <= 2e-2 * max(1.0, abs(lr)), (ln, lr)
    g_nat, g_ref = t_nat.dense.grad, t_ref.dense.grad
    rel = float((g_nat - g_ref).norm() / (g_ref.norm() + 1e-12))
    assert rel < 6e-2, rel
    # a few optimizer steps train without errors
    for _ in range(3):
        t_nat.train_step(batch)
    torch.cuda.synchronize()
    check_error_word(0)
