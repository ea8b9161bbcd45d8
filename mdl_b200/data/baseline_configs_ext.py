"""Benchmark workloads 3-5 (MDL, OneTrans, LONGER/STCA) as reference-schema configs.

Workload 4, OneTrans:

* one behaviour sequence of 512 events (``behavior``): item id Zipf over 1e7
  plus 4 side ids over 1e5, all embedding dim 64, fused into S tokens by a
  320 -> 1024 -> 256 projection MLP (one sequence group, so no SEP token);
* 32 NS tokens from the 300 fields + 64 dense features of workload 2
  (``auto_split``: one MLP from the concatenated inputs to 32 x 256);
* d=256, 8 heads (head_dim 32), FFN 1024, 6 layers, causal attention, pyramid
  that halves the queried S tokens every 2 layers (512, 256, 256, 128, 128, 64);
* one click head (hidden 1024) at positive rate 0.05; batch 1024 per GPU, bf16.

Workload 3, MDL on the RankMixer backbone of workload 2:

* the 300 fields + 64 dense features of workload 2 form the feature tokens
  (T=16, D=768, 2 layers, FFN x4);
* a scene id uniform over 5 scenes (``scene_id``, embedding scope
  ``scenario``) feeds the scenario tokens: 4 tokens per scene plus the global
  token (``tokens_per_scenario: 4``);
* one prior feature per scene (``prior_scene<i>``, scope ``scenario``) and one
  per task (``prior_<task>``, scope ``task``) are the token-unique priors of each
  scenario / task token;
* scene-conditioned feature bias (FiLM on the feature tokens);
* click / like / finish heads at positive rates 0.08 / 0.02 / 0.3, whose
  ground truth depends on the scene;
* batch 2048 per GPU, bf16.
"""

from __future__ import annotations

import copy

from .baseline_configs import _config2_features, _rankmixer_common
from .synthetic import FieldSpec, SequenceSpec, SyntheticSpec

MDL_TASKS = {"click": 0.08, "like": 0.02, "finish": 0.3}
MDL_SCENES = 5


def config3(num_fields: int = 300, batch: int = 2048, tokens_per_scenario: int = 4,
            scene_feature_bias: str = "film") -> tuple[dict, SyntheticSpec]:
    tasks = dict(MDL_TASKS)
    m = _rankmixer_common("mdl_rankmixer", tasks, batch, "bf16", "cuda")
    feats, fields = _config2_features(num_fields)
    feats = copy.deepcopy(feats)
    fields = dict(fields)
    m["features"] = feats
    scenes = _add_mdl_domains(m, feats, fields, tasks, tokens_per_scenario)
    m["tokenization"] = {
        "feature_tokenizer": "rankmixer",
        "num_feature_tokens": 16,
        "scenario_tokens": _scenario_tokens(scenes),
        "task_tokens": _task_tokens(tasks),
    }
    m["model"].update({"embedding_dim": 64, "token_dim": 768, "num_layers": 2, "num_heads": 12, "hidden_dim": 3072,
                       "task_head_hidden_dim": 1536, "ffn_activation": "gelu", "scene_feature_bias": scene_feature_bias,
                       "mdl_feature_interaction": "residual_ffn"})
    m["training"].update({"lr_dense": 1e-4, "lr_sparse": 0.05, "dense_optimizer": "rmsprop", "lr_warmup_steps": 1000,
                          "rmsprop_alpha": 0.99999, "adagrad_initial_accumulator_value": 0.0})
    spec = SyntheticSpec(fields=fields, dense_width=64, task_rates=list(tasks.values()), zipf_s=1.05, seed=0,
                         num_scenarios=MDL_SCENES, scene_field="scene_id", scene_effect=0.5)
    return m, spec


def _scenario_tokens(scenes: list[str]) -> list[dict]:
    return ([{"name": s, "important_inputs": ["scene_id"], "prior_inputs": [f"prior_{s}"]} for s in scenes]
            + [{"name": "global", "important_inputs": ["scene_id"]}])


def _task_tokens(tasks: dict) -> list[dict]:
    return [{"name": t, "important_inputs": [f"prior_{t}"], "prior_inputs": [f"prior_{t}"]} for t in tasks]


def _add_mdl_domains(m: dict, feats: list[dict], fields: dict, tasks: dict, tokens_per_scenario: int) -> list[str]:
    """Scene id (scope ``scenario``) and one prior per task (scope ``task``) as the
    inputs of the scenario / task tokens; returns the scene names."""

    scenes = [f"scene{i}" for i in range(MDL_SCENES)]
    feats.append({"name": "scene_id", "kind": "categorical", "source": "scene_id", "embedding_dim": 64,
                  "embedding_scope": "scenario", "encoding": {"type": "identity", "max_id": MDL_SCENES}})
    fields["scene_id"] = FieldSpec(vocab=MDL_SCENES)
    # one scenario-scoped prior per scene (the reference requires a token-unique prior
    # for every scenario token once there are several scenes)
    for s in scenes:
        name = f"prior_{s}"
        feats.append({"name": name, "kind": "categorical", "source": name, "embedding_dim": 64,
                      "embedding_scope": "scenario", "encoding": {"type": "identity", "max_id": 1000}})
        fields[name] = FieldSpec(vocab=1000)
    for task in tasks:
        name = f"prior_{task}"
        feats.append({"name": name, "kind": "categorical", "source": name, "embedding_dim": 64,
                      "embedding_scope": "task", "encoding": {"type": "identity", "max_id": 1000}})
        fields[name] = FieldSpec(vocab=1000)
    m["scenarios"] = {"names": scenes, "source": "scene_id"}
    m["model"].update({"use_task_tokens": True, "use_scenario_tokens": True, "use_global_scenario_token": True,
                       "use_task_feature_interaction": True, "use_scenario_feature_interaction": True,
                       "tokens_per_scenario": tokens_per_scenario, "mdl_token_state": "coupled"})
    return scenes


def config4(num_fields: int = 300, batch: int = 1024, seq_len: int = 512, side_fields: int = 4,
            item_vocab: int = 10_000_000, side_vocab: int = 100_000, num_layers: int = 6,
            pyramid_schedule: str = "halve", mdl: bool = False) -> tuple[dict, SyntheticSpec]:
    """Workload 4; ``mdl=True`` gives its MDL variant (``mdl_onetrans``): the scene id
    and task priors of workload 3 feed 5 x 1 + 1 scenario tokens and 3 task tokens that
    read the NS tokens after every layer, click / like / finish heads."""

    tasks = dict(MDL_TASKS) if mdl else {"click": 0.05}
    m = _rankmixer_common("mdl_onetrans" if mdl else "onetrans", tasks, batch, "bf16", "cuda")
    feats, fields = _config2_features(num_fields)
    feats = copy.deepcopy(feats)
    fields = dict(fields)
    m["features"] = feats
    seq_fields = [{"name": "item_id", "kind": "categorical", "source": "behavior_item_id", "embedding_dim": 64,
                   "encoding": {"type": "identity", "max_id": item_vocab}}]
    seq_fields += [{"name": f"side{k}", "kind": "categorical", "source": f"behavior_side{k}", "embedding_dim": 64,
                    "encoding": {"type": "identity", "max_id": side_vocab}} for k in range(side_fields)]
    m["sequences"] = [{"name": "behavior", "fields": seq_fields, "max_length": seq_len, "encoder": "raw",
                       "sequence_order": "oldest_to_newest", "truncation": "tail"}]
    m["tokenization"] = {"feature_tokenizer": "auto_split", "num_feature_tokens": 32,
                         "sequence_tokens": [{"name": "behavior", "inputs": ["behavior"]}]}
    m["model"].update({"embedding_dim": 64, "token_dim": 256, "num_layers": num_layers, "num_heads": 8,
                       "hidden_dim": 1024, "task_head_hidden_dim": 1024, "ffn_activation": "gelu",
                       "ns_tokenizer": "auto_split", "num_ns_tokens": 32, "use_pyramid": True,
                       "pyramid_schedule": pyramid_schedule, "pyramid_halve_every": 2, "pyramid_round_to": 32,
                       "use_sep_tokens": True, "sequence_fusion": "intent_ordered",
                       "max_position_embeddings": seq_len + 32, "use_task_tokens": False,
                       "use_scenario_tokens": False, "use_global_scenario_token": False,
                       "use_task_feature_interaction": False, "use_scenario_feature_interaction": False})
    m["training"].update({"lr_dense": 1e-4, "lr_sparse": 0.05, "dense_optimizer": "rmsprop", "lr_warmup_steps": 1000,
                          "rmsprop_alpha": 0.99999, "adagrad_initial_accumulator_value": 0.0})
    seq = SequenceSpec(fields={"item_id": FieldSpec(vocab=item_vocab),
                               **{f"side{k}": FieldSpec(vocab=side_vocab) for k in range(side_fields)}},
                       max_len=seq_len)
    scene_kw = {}
    if mdl:
        scenes = _add_mdl_domains(m, feats, fields, tasks, 1)
        m["tokenization"]["scenario_tokens"] = _scenario_tokens(scenes)
        m["tokenization"]["task_tokens"] = _task_tokens(tasks)
        m["model"]["experimental_model_acknowledged"] = True
        scene_kw = dict(num_scenarios=MDL_SCENES, scene_field="scene_id", scene_effect=0.5)
    spec = SyntheticSpec(fields=fields, dense_width=64, task_rates=list(tasks.values()), zipf_s=1.05, seed=0,
                         sequences={"behavior": seq}, **scene_kw)
    return m, spec


def config5(num_fields: int = 300, batch: int = 512, seq_len: int = 2000, min_len: int = 100,
            item_vocab: int = 10_000_000, query_tokens: int = 256, self_layers: int = 2, d: int = 256, heads: int = 8,
            sequence_head: str = "mixformer", ns_tokens: int = 32) -> tuple[dict, SyntheticSpec]:
    """Workload 5, LONGER: a behaviour sequence of 100-2000 item ids (padded to 2000,
    shared 64-dim item table with the target item), target-item global token, cross
    block to the last 256 events + the target, 2 self blocks (d=256, 8 heads), then a
    MixFormer-style head over 32 NS tokens from the workload-2 fields (or flattened
    LONGER tokens with ``sequence_head="none"``); click head, batch 512 per GPU."""

    tasks = {"click": 0.05}
    m = _rankmixer_common("longer", tasks, batch, "bf16", "cuda")
    feats, fields = _config2_features(num_fields)
    feats = copy.deepcopy(feats)
    feats.append({"name": "target_item", "kind": "categorical", "source": "target_item", "embedding_dim": 64,
                  "encoding": {"type": "identity", "max_id": item_vocab}})
    fields["target_item"] = FieldSpec(vocab=item_vocab)
    m["features"] = feats
    m["sequences"] = [{"name": "behavior", "max_length": seq_len, "encoder": "longer",
                       "sequence_order": "oldest_to_newest", "truncation": "tail",
                       "fields": [{"name": "item_id", "kind": "categorical", "source": "behavior_item_id",
                                   "embedding_dim": 64,
                                   "encoding": {"type": "identity", "max_id": item_vocab, "share_with": "target_item",
                                                "share_embedding": True}}],
                       "target_inputs": ["target_item"], "longer_dim": d, "longer_num_heads": heads,
                       "longer_hidden_dim": 4 * d, "longer_query_tokens": query_tokens,
                       "longer_self_layers": self_layers, "longer_token_merge": 1,
                       "longer_candidate_global_tokens": 1}]
    m["tokenization"] = {"feature_tokenizer": "auto_split", "num_feature_tokens": ns_tokens,
                         "feature_token_inputs": [f["name"] for f in feats if f["name"] != "target_item"]}
    m["model"].update({"embedding_dim": 64, "token_dim": 64, "num_heads": 2, "hidden_dim": 256,
                       "task_head_hidden_dim": 1024, "ffn_activation": "gelu", "sequence_head": sequence_head,
                       "num_layers": 1, "num_ns_tokens": ns_tokens, "use_task_tokens": False,
                       "use_scenario_tokens": False, "use_global_scenario_token": False})
    m["training"].update({"lr_dense": 1e-4, "lr_sparse": 0.05, "dense_optimizer": "rmsprop", "lr_warmup_steps": 1000,
                          "rmsprop_alpha": 0.99999, "adagrad_initial_accumulator_value": 0.0})
    seq = SequenceSpec(fields={"item_id": FieldSpec(vocab=item_vocab)}, max_len=seq_len, min_len=min_len)
    spec = SyntheticSpec(fields=fields, dense_width=64, task_rates=list(tasks.values()), zipf_s=1.05, seed=0,
                         sequences={"behavior": seq})
    return m, spec


def config(n: int, **kw) -> tuple[dict, SyntheticSpec]:
    if n == 3:
        return config3(**kw)
    if n == 4:
        return config4(**kw)
    if n == 5:
        return config5(**kw)
    raise ValueError(f"no benchmark workload {n}")
