"""The benchmark workloads as reference-schema configs plus synthetic-data specs.

``baseline_config(n)`` returns ``(mapping, SyntheticSpec)`` for workload ``n``:

1. tiny RankMixer on CPU/gloo: 16 one-hot fields (vocab 10 000, dim 16), 8 dense,
   T=8, D=64, 2 layers, FFN x4, one click head (rate 0.1), batch 256, row-wise
   Adagrad lr 0.05, Adam lr 1e-3, fp32;
2. RankMixer ~100M+ dense: 300 fields, vocab log-uniform in [1e3, 1e7] (about 200M
   rows), dim 64 fp32 tables, Zipf(1.05) ids, 20% multi-hot (length U[1,20],
   sum pooling), 64 dense, T=16, D=768, 2 layers, FFN x4, click (0.05) and
   conversion (0.01) heads, batch 2048 per GPU, bf16;
3. MDL on a RankMixer backbone (config 2 features), 5 scenes, 4 domain tokens
   per scene, scene-conditioned feature bias, click/like/finish heads;
4. OneTrans (sequence 512 with 4 side fields, 32 NS tokens, d=256, 8 heads,
   6 layers, pyramid halving every 2 layers), batch 1024;
5. LONGER/STCA (sequence U[100, 2000] padded to 2000, target attention to 256,
   2 self layers) feeding a MixFormer-style head, batch 512.

The mappings go through the same loader as YAML files, so they are ordinary
configs; ``write_baseline_yamls`` dumps them under ``configs/``.
"""

from __future__ import annotations

import math

import numpy as np

from .synthetic import FieldSpec, SyntheticSpec


def _vocabs(n: int, lo: float, hi: float, target_total: float, seed: int = 0) -> list[int]:
    """Per-field log-uniform vocab sizes; the first seed whose total is within 5% of target."""

    for s in range(seed, seed + 10000):
        rng = np.random.default_rng(s)
        v = np.exp(rng.uniform(math.log(lo), math.log(hi), size=n)).astype(np.int64)
        if abs(v.sum() - target_total) <= 0.05 * target_total:
            return [int(x) for x in v]
    raise RuntimeError("no vocab draw near the target total")


def _rankmixer_common(name: str, tasks: dict[str, float], batch: int, precision: str, device: str) -> dict:
    return {
        "runtime": {"device": device, "precision": precision, "distributed": "none", "attention_backend": "flash"},
        "data": {"train": {"format": "flat_parquet", "inputs": [], "labels": {t: t for t in tasks}}},
        "model": {"name": name},
        "training": {
            "batch_size": batch,
            "embedding_distribution": "sharded",
            "embedding_sharding": {"strategy": "auto", "table_wise_max_rows": 65536},
            "sparse_optimizer": "rowwise_adagrad",
            "embedding_weight_dtype": "fp32",
            "loss_reduction": "mean_per_task",
            "lr_warmup_steps": 0,
            "save_checkpoint": False,
            "fixed_test_eval": {"enabled": False},
        },
    }


def config1() -> tuple[dict, SyntheticSpec]:
    tasks = {"click": 0.1}
    m = _rankmixer_common("rankmixer", tasks, 256, "fp32", "cpu")
    feats = [{"name": f"c{i}", "kind": "categorical", "source": f"c{i}", "embedding_dim": 16,
              "encoding": {"type": "identity", "max_id": 10000}} for i in range(16)]
    feats.append({"name": "dense", "kind": "dense", "source": "dense", "dimension": 8, "presence": False})
    m["features"] = feats
    m["tokenization"] = {"feature_tokenizer": "rankmixer", "num_feature_tokens": 8}
    m["model"].update({"embedding_dim": 16, "token_dim": 64, "num_layers": 2, "num_heads": 4, "hidden_dim": 256,
                       "task_head_hidden_dim": 64, "ffn_activation": "gelu"})
    m["training"].update({"lr_dense": 1e-3, "lr_sparse": 0.05, "dense_optimizer": "adam",
                          "adagrad_initial_accumulator_value": 0.0, "adagrad_eps": 1e-10})
    spec = SyntheticSpec(fields={f"c{i}": FieldSpec(vocab=10000) for i in range(16)}, dense_width=8,
                         task_rates=list(tasks.values()), zipf_s=None, seed=0)
    return m, spec


def _config2_features(num_fields: int = 300, seed: int = 0) -> tuple[list[dict], dict[str, FieldSpec]]:
    vocabs = _vocabs(num_fields, 1e3, 1e7, 2.0e8 * num_fields / 300.0, seed)
    rng = np.random.default_rng(seed + 1)
    multi = set(rng.choice(num_fields, size=num_fields // 5, replace=False).tolist())
    feats, fields = [], {}
    for i in range(num_fields):
        name = f"f{i:03d}"
        is_multi = i in multi
        feat = {"name": name, "kind": "categorical", "source": name, "embedding_dim": 64,
                "encoding": {"type": "identity", "max_id": vocabs[i]}, "pooling": "sum" if is_multi else "none"}
        if is_multi:
            feat["max_length"] = 20
        feats.append(feat)
        fields[name] = FieldSpec(vocab=vocabs[i], multi_hot=is_multi, min_len=1, max_len=20 if is_multi else 1)
    feats.append({"name": "dense", "kind": "dense", "source": "dense", "dimension": 64, "presence": False})
    return feats, fields


def config2(num_fields: int = 300, batch: int = 2048) -> tuple[dict, SyntheticSpec]:
    tasks = {"click": 0.05, "conversion": 0.01}
    m = _rankmixer_common("rankmixer", tasks, batch, "bf16", "cuda")
    feats, fields = _config2_features(num_fields)
    m["features"] = feats
    m["tokenization"] = {"feature_tokenizer": "rankmixer", "num_feature_tokens": 16}
    m["model"].update({"embedding_dim": 64, "token_dim": 768, "num_layers": 2, "num_heads": 12, "hidden_dim": 3072,
                       "task_head_hidden_dim": 1536, "ffn_activation": "gelu"})
    # RMSprop is the reference's only dense optimizer; both benchmark arms use it.
    m["training"].update({"lr_dense": 1e-4, "lr_sparse": 0.05, "dense_optimizer": "rmsprop", "lr_warmup_steps": 1000,
                          "rmsprop_alpha": 0.99999, "adagrad_initial_accumulator_value": 0.0})
    spec = SyntheticSpec(fields=fields, dense_width=64, task_rates=list(tasks.values()), zipf_s=1.05, seed=0)
    return m, spec


def baseline_config(n: int, **kw) -> tuple[dict, SyntheticSpec]:
    if n == 1:
        return config1()
    if n == 2:
        return config2(**kw)
    from . import baseline_configs_ext

    return baseline_configs_ext.config(n, **kw)


def scaled_config(n: int, scale: float, **kw) -> tuple[dict, SyntheticSpec]:
    """A proportionally smaller workload (tests / smoke): vocabularies scaled by ``scale``."""

    m, spec = baseline_config(n, **kw)
    for f in m["features"]:
        enc = f.get("encoding")
        if enc and enc.get("max_id"):
            enc["max_id"] = max(16, int(enc["max_id"] * scale))
    for name, fs in spec.fields.items():
        fs.vocab = max(16, int(fs.vocab * scale))
    for seq in m.get("sequences", []):
        for fl in seq.get("fields", []):
            enc = fl.get("encoding")
            if enc and enc.get("max_id"):
                enc["max_id"] = max(16, int(enc["max_id"] * scale))
    for ss in (spec.sequences or {}).values():
        for fs in ss.fields.values():
            fs.vocab = max(16, int(fs.vocab * scale))
    return m, spec
