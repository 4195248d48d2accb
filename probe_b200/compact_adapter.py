"""Compact heterogeneous LoRA adapters on disk, and their packing into the flat
tables the segmented kernels read.

Drop-in for ``loraforge_kernels.compact_adapter`` (compact_adapter.py:1-145)
and the bucketing tool (bucket_adapter_ranks.py:1-68), plus the step the
reference leaves to its serving code: loading several compact adapters and
packing one module's factors into ``a_flat [sum r, K]``, ``b_flat [sum r, N]``
(scale folded in, rank-major), ``offsets`` and ``ranks`` -- the tables of
``segmented_branch_varlen`` / ``ragged_branch.branch`` / ``lora_sgmv_*``.

Compaction is a storage transformation, not a truncation: an adapter already
zero-padded to its allocated ranks is cut to exactly those ranks, and the cut
is refused when a discarded coordinate is live in both factors.  Rank-0
targets disappear (the layer runs its base linear alone).
"""

from __future__ import annotations

import copy
import json
import math
import re
from pathlib import Path

import torch

_A_SUFFIX = ".lora_A.weight"
_B_SUFFIX = ".lora_B.weight"


def module_name(a_key: str) -> str:
    """PEFT module name of a ``...lora_A.weight`` key (compact_adapter.py:20-24)."""
    if not a_key.endswith(_A_SUFFIX):
        raise ValueError(f"Expected a PEFT Linear LoRA key: {a_key}")
    name = a_key[: -len(_A_SUFFIX)]
    return name[len("base_model.model."):] if name.startswith("base_model.model.") else name


def pattern_value(config: dict, field: str, default: str, name: str):
    """PEFT's rank/alpha pattern lookup: the first pattern that matches a suffix
    of the module name (anchored at a dot or the start), else the default
    (compact_adapter.py:27-32)."""
    for pattern, value in config.get(field, {}).items():
        if re.match(rf"(.*\.)?({pattern})$", name):
            return value
    return config[default]


def lora_scale(config: dict, name: str) -> float:
    """alpha / r, or alpha / sqrt(r) for rsLoRA, with the per-module patterns."""
    rank = int(pattern_value(config, "rank_pattern", "r", name))
    alpha = float(pattern_value(config, "alpha_pattern", "lora_alpha", name))
    return alpha / (math.sqrt(rank) if config.get("use_rslora") else rank)


def _check_plain_lora(config: dict):
    unsupported = (config.get("peft_type", "LORA") != "LORA" or config.get("use_dora") or config.get("lora_bias")
                   or config.get("bias", "none") != "none" or config.get("modules_to_save")
                   or config.get("target_parameters") or config.get("layer_replication")
                   or config.get("use_qalora") or config.get("alora_invocation_tokens"))
    if unsupported:
        raise ValueError("Compaction currently supports ordinary bias-free Linear LoRA/rsLoRA only")


def compact_zero_padded(tensors: dict, config: dict, ranks):
    """(compact tensors, compact config, manifest) for zero-padded factors cut to
    ``ranks`` (one per A/B pair, in sorted key order; compact_adapter.py:35-110).

    The compact config pins every kept module's rank and an alpha that keeps its
    scale exactly (``scale * r`` or ``scale * sqrt(r)``); rank-0 modules are
    dropped.  Each kept module is checked in fp64 on a fixed random probe.
    """
    _check_plain_lora(config)
    keys = sorted(k for k in tensors if k.endswith(_A_SUFFIX))
    if not keys or len(ranks) != len(keys):
        raise ValueError(f"Allocation has {len(ranks)} ranks for {len(keys)} A/B pairs")
    out = {}
    cfg = copy.deepcopy(config)
    cfg.update(rank_pattern={}, alpha_pattern={}, target_modules=[], layers_to_transform=None,
               layers_pattern=None, exclude_modules=None, inference_mode=True)
    layers, seen = [], set()
    probe_gen = torch.Generator().manual_seed(91)
    for a_key, rank in zip(keys, ranks):
        b_key = a_key[: -len(_A_SUFFIX)] + _B_SUFFIX
        a, b = tensors[a_key], tensors[b_key]
        if a.ndim != 2 or b.ndim != 2 or a.shape[0] != b.shape[1]:
            raise ValueError(f"Unsupported factor shapes for {a_key}")
        if isinstance(rank, bool) or not isinstance(rank, int) or not 0 <= rank <= a.shape[0]:
            raise ValueError(f"Invalid retained rank {rank} for {a_key}")
        # a coordinate can go only if one of its two factors is zero
        live = a[rank:].ne(0).any(dim=1) & b[:, rank:].ne(0).any(dim=0)
        if bool(live.any()):
            raise ValueError(f"{a_key}: discarded coordinates are nonzero; truncate before compacting")
        if not (torch.isfinite(a).all() and torch.isfinite(b).all()):
            raise ValueError(f"Nonfinite factors: {a_key}")
        name = module_name(a_key)
        nominal = int(pattern_value(config, "rank_pattern", "r", name))
        if nominal != a.shape[0]:
            raise ValueError(f"{name}: config rank {nominal} != tensor rank {a.shape[0]}")
        scale = lora_scale(config, name)
        ca, cb = a[:rank].contiguous(), b[:, :rank].contiguous()
        probe = torch.randn(3, a.shape[1], generator=probe_gen, dtype=torch.float64)
        want = scale * ((probe @ a.double().T) @ b.double().T)
        got = scale * ((probe @ ca.double().T) @ cb.double().T)
        torch.testing.assert_close(got, want, rtol=1e-10, atol=1e-12)
        if rank:
            cfg["target_modules"].append(name)
            cfg["rank_pattern"][re.escape(name)] = rank
            cfg["alpha_pattern"][re.escape(name)] = scale * (math.sqrt(rank) if config.get("use_rslora") else rank)
            out[a_key], out[b_key] = ca, cb
        seen.update((a_key, b_key))
        layers.append(dict(module=name, a_key=a_key, b_key=b_key, rank=rank, original_rank=nominal, scale=scale,
                           a_shape=list(ca.shape), b_shape=list(cb.shape),
                           max_abs_error_fp64=float((got - want).abs().max()),
                           padded_elements=a.numel() + b.numel(), compact_elements=ca.numel() + cb.numel()))
    if set(tensors) != seen:
        raise ValueError("Unrecognized/non-LoRA tensors; refusing to silently drop additional adapter state")
    manifest = dict(base_only=not out, validation_passed=True, layers=layers, original_modules=len(keys),
                    active_modules=sum(d["rank"] > 0 for d in layers),
                    zero_modules=sum(d["rank"] == 0 for d in layers),
                    original_rank_sum=sum(d["original_rank"] for d in layers), compact_rank_sum=sum(ranks),
                    padded_elements=sum(d["padded_elements"] for d in layers),
                    compact_elements=sum(d["compact_elements"] for d in layers))
    return out, cfg, manifest


def export_compact(source, output, ranks) -> dict:
    """Write the compact adapter of directory ``source`` to the new directory
    ``output`` (compact_adapter.py:113-127); returns the manifest."""
    from safetensors import safe_open
    from safetensors.torch import load_file, save_file

    source, output = Path(source), Path(output)
    if source.resolve() == output.resolve() or output.exists():
        raise ValueError("Output must be a new directory distinct from the source")
    weights = load_file(source / "adapter_model.safetensors")
    config = json.loads((source / "adapter_config.json").read_text())
    compact, cfg, manifest = compact_zero_padded(weights, config, ranks)
    with safe_open(source / "adapter_model.safetensors", framework="pt") as handle:
        metadata = handle.metadata()
    output.mkdir(parents=True)
    if compact:
        save_file(compact, output / "adapter_model.safetensors", metadata=metadata)
        (output / "adapter_config.json").write_text(json.dumps(cfg, indent=2) + "\n")
    manifest["source"] = str(source.resolve())
    (output / "compaction.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def bucket_rank(rank: int, maximum: int = 32) -> int:
    """The power of two covering ``rank``, capped at ``maximum`` (bucket_adapter_ranks.py:13-14)."""
    return min(maximum, 1 << (rank - 1).bit_length())


def bucket_zero_pad(tensors: dict, config: dict, maximum: int = 32):
    """Zero-pad every module to its rank bucket (bucket_adapter_ranks.py:17-60):
    (padded tensors, config with the new rank_pattern, per-module report).
    Exact: the padded coordinates are zero in both factors."""
    pattern = config.get("rank_pattern", {})
    new_pattern = dict(pattern)
    out = dict(tensors)
    report = []
    for a_key in sorted(k for k in tensors if k.endswith(_A_SUFFIX)):
        b_key = a_key[: -len(_A_SUFFIX)] + _B_SUFFIX
        a, b = tensors[a_key], tensors[b_key]
        old = a.shape[0]
        if old > maximum:
            raise ValueError(f"{a_key}: rank {old} is above the largest bucket {maximum}")
        new = bucket_rank(old, maximum)
        if new != old:
            pa = a.new_zeros((new, a.shape[1]))
            pb = b.new_zeros((b.shape[0], new))
            pa[:old].copy_(a)
            pb[:, :old].copy_(b)
            out[a_key], out[b_key] = pa, pb
        name = a_key[: -len(_A_SUFFIX)]
        matches = [key for key in pattern if name.endswith(key)]
        if len(matches) != 1:
            raise RuntimeError(f"cannot map tensor module to rank_pattern: {name}")
        new_pattern[matches[0]] = new
        report.append({"module": matches[0], "old_rank": old, "new_rank": new})
    cfg = dict(config, rank_pattern=new_pattern)
    return out, cfg, report


def pack_sgmv_tables(factors, device="cuda", dtype=torch.bfloat16):
    """Flat tables of one layer for adapters ``factors[i] = (A [r_i, K], B [N, r_i], scale_i)``
    (``None`` or r_i = 0: no LoRA for adapter i).

    Returns ``(a_flat [sum r, K], b_flat [sum r, N], offsets [n], ranks [n])``:
    adapter i's rows are ``offsets[i] .. offsets[i] + ranks[i]``, its B is stored
    rank-major with the scale folded in (the layout ``ragged_branch.branch`` and
    ``segmented_branch_varlen`` read, ragged_branch.py:30-33).
    """
    ks = {f[0].shape[1] for f in factors if f is not None and f[0].shape[0] > 0}
    ns = {f[1].shape[0] for f in factors if f is not None and f[0].shape[0] > 0}
    if len(ks) > 1 or len(ns) > 1:
        raise ValueError("all adapters of a layer must share K and N")
    k = ks.pop() if ks else 0
    n = ns.pop() if ns else 0
    ranks = [0 if f is None else int(f[0].shape[0]) for f in factors]
    offsets, total = [], 0
    for r in ranks:
        offsets.append(total)
        total += r
    a_flat = torch.zeros((max(total, 1), k), dtype=torch.float64)
    b_flat = torch.zeros((max(total, 1), n), dtype=torch.float64)
    for f, off, r in zip(factors, offsets, ranks):
        if r == 0:
            continue
        a, b, scale = f
        if b.shape[1] != r:
            raise ValueError("lora_B must be [N, r] with the rank of lora_A")
        a_flat[off:off + r] = a.double()
        b_flat[off:off + r] = b.double().T * float(scale)
    return (a_flat.to(device, dtype), b_flat.to(device, dtype),
            torch.tensor(offsets, dtype=torch.int64, device=device),
            torch.tensor(ranks, dtype=torch.int64, device=device))


def load_sgmv_tables(adapter_dirs, module: str, device="cuda", dtype=torch.bfloat16):
    """Read one module's factors from several adapter directories (PEFT layout,
    compact or not) and pack them with ``pack_sgmv_tables``; adapter i is
    ``adapter_dirs[i]``.  An adapter without the module (e.g. a compact adapter
    whose module was cut to rank 0) gets rank 0."""
    from safetensors.torch import load_file

    factors = []
    for d in adapter_dirs:
        d = Path(d)
        weights_path = d / "adapter_model.safetensors"
        if not weights_path.exists():  # base only (every module cut to rank 0)
            factors.append(None)
            continue
        weights = load_file(weights_path)
        config = json.loads((d / "adapter_config.json").read_text())
        hit = [k for k in weights if k.endswith(_A_SUFFIX) and module_name(k) == module]
        if not hit:
            factors.append(None)
            continue
        a = weights[hit[0]]
        b = weights[hit[0][: -len(_A_SUFFIX)] + _B_SUFFIX]
        factors.append((a, b, lora_scale(config, module)))
    return pack_sgmv_tables(factors, device=device, dtype=dtype)
