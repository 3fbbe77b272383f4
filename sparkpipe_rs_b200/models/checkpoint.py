"""Model checkpoints as stage packs (csrc/core/stagepack.{h,cpp}).

``save_pack`` writes a model's weight dict into a pack directory: every tensor as
one 4 KiB-aligned region, block-scaled fp8 weights as two tensors (``<name>.q``
e4m3 values, ``<name>.s`` fp32 scales), and the model configuration in the index
metadata. ``load_pack`` reads it back onto a device, optionally only what one rank
holds: an expert-parallel rank's routed experts (a leading-row range of each expert
stack, plus the shared experts) or a tensor-parallel rank's shard (the TP shard
engine's view, read strided from the file). Reads go through pinned host buffers
and one host-to-device copy per tensor.

Reference: the stage-pack resolve contract and the shard read of
crates/spark-abi/vendor/sparkpipe/model-families/glm52/include/sparkpipe/
spark_glm52_stagepack.h:11-52 and include/sparkpipe/spark_tp_shard.h:132-148; the
MoE pack validation of crates/spark-node/src/rank_daemon/ring_runtime.rs:804.
"""
from __future__ import annotations

import json

import torch

from ..core import core
from .config import MLAMoEConfig

_DTYPES = {torch.bfloat16: "BF16", torch.float32: "F32", torch.float16: "F16", torch.int32: "I32",
           torch.float8_e4m3fn: "F8_E4M3", torch.uint8: "U8"}
_BY_NAME = {v: k for k, v in _DTYPES.items()}
# configuration fields a pack must agree on with the model it is loaded into
_SHAPE_FIELDS = ("num_layers", "hidden_size", "num_heads", "q_lora_rank", "kv_lora_rank", "qk_nope_head_dim",
                 "qk_rope_head_dim", "v_head_dim", "n_routed_experts", "n_shared_experts", "moe_intermediate_size",
                 "intermediate_size", "vocab_size", "weight_dtype")


def _fp8_type():
    from .. import ops

    return ops.Fp8Weight


def save_pack(root, cfg: MLAMoEConfig, weights: dict, model_id: str | None = None) -> int:
    """Writes ``weights`` (name -> tensor or Fp8Weight) as a stage pack; returns the
    tensor bytes written."""
    Fp8 = _fp8_type()
    meta = {"config": {k: getattr(cfg, k) for k in _SHAPE_FIELDS if hasattr(cfg, k)},
            "config_name": cfg.name, "fp8_scale_rows": {}}
    parts = []
    for name, t in weights.items():
        if isinstance(t, Fp8):
            parts += [(name + ".q", t.q), (name + ".s", t.s)]
            meta["fp8_scale_rows"][name] = int(t.sa_rows)
        else:
            parts.append((name, t))
    w = core().stagepack.Writer(str(root), model_id or cfg.name, json.dumps(meta))
    for name, t in parts:
        x = t.detach().contiguous().cpu()
        if x.dtype not in _DTYPES:
            raise TypeError(f"{name}: dtype {x.dtype} has no pack encoding")
        w.add(name, _DTYPES[x.dtype], list(x.shape), x.element_size(), x.data_ptr(), x.numel() * x.element_size())
    w.finish()
    return int(w.bytes_written)


def _check_config(meta: dict, cfg: MLAMoEConfig):
    stored = meta.get("config", {})
    diff = [k for k in _SHAPE_FIELDS if k in stored and hasattr(cfg, k) and stored[k] != getattr(cfg, k)]
    if diff:
        raise ValueError(f"stage pack was written for another model shape: {diff}")


def _host(shape, dtype, pinned: bool):
    return torch.empty(shape, dtype=dtype, pin_memory=pinned)


def load_pack(root, cfg: MLAMoEConfig, device="cpu", experts: tuple[int, int] | None = None,
              tp: tuple[int, int] | None = None, layers: list[int] | None = None, verify: bool = False) -> dict:
    """Weights of ``cfg`` from a stage pack, on ``device``. ``experts`` = (lo, hi): only
    routed experts lo..hi-1 (plus every shared expert) of the expert stacks, as an
    expert-parallel rank holds them. ``tp`` = (degree, rank): this rank's shard of every
    tensor (bf16 / fp32 packs). ``layers``: only these decoder layers. ``verify``
    checks each whole-tensor read against its stored fingerprint."""
    S = core().stagepack
    pk = S.Pack.open(str(root))
    meta = json.loads(pk.metadata)
    _check_config(meta, cfg)
    dev = torch.device(device)
    pinned = dev.type == "cuda"
    Fp8 = _fp8_type()
    names = pk.names()
    logical = []
    for n in names:
        base = n[:-2] if n.endswith((".q", ".s")) and n[:-2] in meta.get("fp8_scale_rows", {}) else n
        if base not in logical:
            logical.append(base)
    if tp is not None and meta.get("fp8_scale_rows"):
        raise ValueError("tensor-parallel shards are read from bf16 / fp32 packs")
    if tp is not None:
        from ..parallel.tensor_parallel import geometry

        T = core().tp
        shape_desc, geo = T.Shape(tp[0], tp[1], 1, 0), geometry(cfg)

    def read(name):
        e = pk.entry(name)
        dtype, shape = _BY_NAME[e["dtype"]], list(e["shape"])
        if experts is not None and name.split(".")[-2 if name.endswith((".q", ".s")) else -1] in ("e_w13", "e_w2"):
            lo, hi = experts
            E = cfg.n_routed_experts
            out = _host([(hi - lo) + (shape[0] - E)] + shape[1:], dtype, pinned)
            row = out[0].numel() * out.element_size()
            pk.read_rows(name, lo, hi - lo, out.data_ptr(), (hi - lo) * row)
            if shape[0] > E:
                pk.read_rows(name, E, shape[0] - E, out[hi - lo:].data_ptr(), (shape[0] - E) * row)
        elif tp is not None:
            view = T.compute_view(T.TensorSpec(name, shape, torch.empty((), dtype=dtype).element_size()),
                                  shape_desc, geo)
            if view.shard_class != T.ShardClass.REPLICATED:
                shape[view.split_dimension] = sum(ext for _, ext in view.ranges)
            out = _host(shape, dtype, pinned)
            pk.read_shard(name, shape_desc, geo, out.data_ptr(), out.numel() * out.element_size())
        else:
            out = _host(shape, dtype, pinned)
            pk.read(name, out.data_ptr(), out.numel() * out.element_size(), verify)
        return out.to(dev, non_blocking=True) if dev.type != "cpu" else out

    w = {}
    for name in logical:
        if layers is not None and name.startswith("l") and "." in name:
            if int(name[1:name.index(".")]) not in layers:
                continue
        if name in meta.get("fp8_scale_rows", {}):
            w[name] = Fp8(read(name + ".q"), read(name + ".s"), int(meta["fp8_scale_rows"][name]))
        else:
            w[name] = read(name)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    return w


def pack_config_fields(root) -> dict:
    """The model-shape fields a pack was written with (from its index)."""
    return json.loads(core().stagepack.Pack.open(str(root)).metadata).get("config", {})


__all__ = ["save_pack", "load_pack", "pack_config_fields"]
