"""Attention preflight: before any data is read, check that every attention a config
will run has a kernel here, and describe which (reference ``_attention_runtime_description``
/ ``_requires_varlen_attention``, ``src/train.py:314-440``).

* OneTrans mixed causal attention and LONGER cross / self attention run the
  tcgen05 flash attention (``csrc/fmha.cu``): head_dim 32, sm_100 devices;
* MDL domain-aware attention and the task-query readout run the few-query kernel
  when both token counts are at most 64 (PyTorch SDPA beyond);
* MixFormer / STCA single-query attention and the MDL-OneTrans sequence reader
  are batched products in PyTorch.
"""

from __future__ import annotations

import torch


def _fmha_check(name: str, dim: int, heads: int, problems: list[str]) -> str:
    if heads <= 0 or dim % heads or dim // heads != 32:
        problems.append(f"{name}: the flash attention kernel needs head_dim 32 (d={dim}, heads={heads})")
    return "tcgen05 flash attention (head_dim 32)"


def attention_preflight(config, device: torch.device | str | None = None) -> dict:
    """``{"paths": {...}}``; raises ``ValueError`` listing every unsupported attention."""

    m = config.model
    paths: dict[str, str] = {}
    problems: list[str] = []
    if m.name in ("onetrans", "mdl_onetrans"):
        paths["mixed_causal"] = _fmha_check("OneTrans", int(m.token_dim), int(m.num_heads), problems)
    for seq in config.sequences:
        if seq.encoder == "longer":
            d = int(seq.longer_dim)
            heads = int(seq.longer_num_heads or max(1, d // 32))
            paths[f"longer:{seq.name}"] = _fmha_check(f"LONGER {seq.name}", d, heads, problems)
        elif seq.encoder == "stca":
            paths[f"stca:{seq.name}"] = "single-query attention (PyTorch batched products)"
    if m.name in ("mixformer", "mdl_mixformer") or getattr(m, "sequence_head", "none") == "mixformer":
        paths["mixformer_cross"] = "reordered single-query attention (PyTorch batched products)"
    if m.name.startswith("mdl_"):
        res = config.resolved.tokenization
        nq = max(len(res.scenario_token_specs), len(res.task_token_specs))
        paths["domain"] = "few-query kernel" if nq <= 64 else "PyTorch SDPA (more than 64 domain tokens)"
        if m.name == "mdl_onetrans" and m.first_domain_sequence_layer is not None:
            paths["domain_sequence"] = "masked attention over [Q_S; NS] (PyTorch batched products)"
    dev = torch.device(device) if device is not None else None
    if dev is not None and dev.type == "cuda" and any("flash" in p for p in paths.values()):
        major, minor = torch.cuda.get_device_capability(dev)
        if major != 10:
            problems.append(f"the flash attention kernel is built for sm_100a; device is sm_{major}{minor}")
    if problems:
        raise ValueError("attention preflight failed: " + "; ".join(problems))
    return {"paths": paths}
