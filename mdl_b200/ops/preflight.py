"""Attention preflight: before any data is read, check that every attention a config
will run has a kernel here, and describe which (reference ``_attention_runtime_description``
/ ``_requires_varlen_attention``, ``src/train.py:314-440``).

* OneTrans mixed causal attention and LONGER cross / self / inner attention run the
  tcgen05 flash attention (``csrc/fmha.cu``) for head_dim 32 and the CUDA-core kernels
  (``csrc/attn_simt.cu``) for head_dim 8, 16 and 64, on sm_100 devices (any width with
  ``runtime.kernel_backend: torch``);
* MDL domain-aware attention and the task-query readout run the few-query kernel
  when both token counts are at most 64 (PyTorch SDPA beyond);
* MixFormer / STCA single-query attention and the MDL-OneTrans sequence reader
  are batched products in PyTorch.
"""

from __future__ import annotations

import torch


def _fmha_check(name: str, dim: int, heads: int, problems: list[str], backend: str = "native") -> str:
    from .attention import NATIVE_HEAD_DIMS

    if heads <= 0 or dim % heads:
        problems.append(f"{name}: width {dim} is not divisible by {heads} heads")
        return "none"
    hd = dim // heads
    if backend == "torch":
        return f"PyTorch attention (head_dim {hd})"
    if hd == 32:
        return "tcgen05 flash attention (head_dim 32)"
    if hd in NATIVE_HEAD_DIMS:
        return f"CUDA-core suffix attention (head_dim {hd})"
    problems.append(f"{name}: the native attention kernels take head_dim {NATIVE_HEAD_DIMS} (d={dim}, "
                    f"heads={heads}); set runtime.kernel_backend: torch")
    return "none"


def attention_preflight(config, device: torch.device | str | None = None) -> dict:
    """``{"paths": {...}}``; raises ``ValueError`` listing every unsupported attention."""

    m = config.model
    paths: dict[str, str] = {}
    problems: list[str] = []
    backend = config.runtime.kernel_backend
    if m.name in ("onetrans", "mdl_onetrans"):
        paths["mixed_causal"] = _fmha_check("OneTrans", int(m.token_dim), int(m.num_heads), problems, backend)
    for seq in config.sequences:
        if seq.encoder == "longer":
            d = int(seq.longer_dim)
            heads = seq.longer_num_heads  # as LongerEncoder resolves it
            if heads is None:
                heads = int(m.num_heads) if d % int(m.num_heads) == 0 else next(h for h in (8, 4, 2, 1) if d % h == 0)
            heads = int(heads)
            merged = d * int(seq.longer_token_merge)
            paths[f"longer:{seq.name}"] = _fmha_check(f"LONGER {seq.name}", merged, heads, problems, backend)
            if int(seq.longer_inner_layers):
                paths[f"longer_inner:{seq.name}"] = _fmha_check(f"LONGER {seq.name} inner", d, heads, problems,
                                                                backend)
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
    if dev is not None and dev.type == "cuda" and any("flash" in p or "CUDA-core" in p for p in paths.values()):
        major, minor = torch.cuda.get_device_capability(dev)
        if major != 10:
            problems.append(f"the flash attention kernel is built for sm_100a; device is sm_{major}{minor}")
    if problems:
        raise ValueError("attention preflight failed: " + "; ".join(problems))
    return {"paths": paths}
