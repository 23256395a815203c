"""Hugging Face Llama checkpoints <-> this runtime's weights.

A checkpoint directory holds ``config.json`` and ``*.safetensors`` shards
(the layout ``LlamaForCausalLM.save_pretrained`` writes; Llama 3 / 3.1 /
3.2 and other models of that architecture).  Loading fuses the tensors into
the kernels' layouts on the host, shard by shard, and moves each result to
the device once:

* ``q_proj | k_proj | v_proj`` -> ``wqkv`` [(H + 2 Hkv) * 128, hidden], rows
  in that order (the checkpoint's q/k rows already follow the rotate-half
  RoPE convention the kernels use);
* ``gate_proj``, ``up_proj`` -> ``w13``, rows interleaved in blocks of half
  the SiLU-mul GEMM tile (:func:`connex_b200.ops.interleave_gate_up`);
* ``lm_head`` = ``embed_tokens`` when ``tie_word_embeddings``.

Only layers ``[l0, l1)`` are read for a pipeline stage, plus the embedding
on the first stage and the final norm and LM head on the last.  The
reference serves checkpoints through vLLM / SGLang (its engines load them);
this is the loader of its own runtime.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Dict, Iterable, Optional, Tuple

import torch

from connex_b200 import ops
from connex_b200.models.llama import LayerWeights, LlamaConfig, LlamaWeights

HEAD_DIM = 128          # the attention kernels' head size


def config_from_hf(src) -> LlamaConfig:
    """:class:`LlamaConfig` of an HF ``config.json`` (a path, a directory or a dict)."""
    if isinstance(src, (str, os.PathLike)):
        path = os.path.join(src, "config.json") if os.path.isdir(src) else src
        with open(path) as f:
            src = json.load(f)
    c = dict(src)
    heads = int(c["num_attention_heads"])
    head_dim = int(c.get("head_dim") or c["hidden_size"] // heads)
    if head_dim != HEAD_DIM:
        raise ValueError(f"head_dim {head_dim} is not supported (the attention kernels use {HEAD_DIM})")
    ffn = int(c["intermediate_size"])
    if ffn % (ops.GATE_UP_TILE // 2):
        raise ValueError(f"intermediate_size {ffn} is not a multiple of {ops.GATE_UP_TILE // 2}")
    if c.get("attention_bias") or c.get("mlp_bias"):
        raise ValueError("attention / MLP biases are not supported")
    # older configs: rope_theta + rope_scaling; newer ones: rope_parameters holding both
    rs = c.get("rope_scaling") or c.get("rope_parameters") or None
    scaling = None
    if rs:
        kind = rs.get("rope_type", rs.get("type"))
        if kind == "llama3":
            scaling = (float(rs["factor"]), float(rs["low_freq_factor"]), float(rs["high_freq_factor"]),
                       int(rs["original_max_position_embeddings"]))
        elif kind not in (None, "default"):
            raise ValueError(f"rope_scaling type {kind!r} is not supported")
    theta = c.get("rope_theta")
    if theta is None:
        theta = (c.get("rope_parameters") or {}).get("rope_theta", 10000.0)
    return LlamaConfig(vocab_size=int(c["vocab_size"]), hidden=int(c["hidden_size"]),
                       layers=int(c["num_hidden_layers"]), heads=heads,
                       kv_heads=int(c.get("num_key_value_heads") or heads), head_dim=head_dim, ffn=ffn,
                       rope_theta=float(theta), eps=float(c.get("rms_norm_eps", 1e-5)),
                       max_pos=int(c.get("max_position_embeddings", 8192)), rope_scaling=scaling)


def _tied(src) -> bool:
    if isinstance(src, (str, os.PathLike)):
        with open(os.path.join(src, "config.json")) as f:
            src = json.load(f)
    return bool(src.get("tie_word_embeddings", False))


class _Shards:
    """Name -> tensor reads over the checkpoint's safetensors files."""

    def __init__(self, path: str):
        from safetensors import safe_open
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no *.safetensors in {path}")
        self._open = [safe_open(f, framework="pt", device="cpu") for f in files]
        self.where: Dict[str, object] = {}
        for h in self._open:
            for k in h.keys():
                self.where[k] = h

    def get(self, name: str) -> torch.Tensor:
        h = self.where.get(name)
        if h is None:
            raise KeyError(f"checkpoint has no tensor {name!r}")
        return h.get_tensor(name)

    def has(self, name: str) -> bool:
        return name in self.where


def load_llama(path: str, device, dtype=torch.bfloat16, layers: Optional[Tuple[int, int]] = None,
               cfg: Optional[LlamaConfig] = None, tp: Optional[Tuple[int, int]] = None) -> LlamaWeights:
    """Weights of layers ``[l0, l1)`` (all by default) of the checkpoint in
    ``path``, in the kernels' layouts, on ``device``.  Tensors the stage
    does not own (embedding off the first stage, head off the last) are
    ``None``.  ``tp = (rank, world)`` keeps only that tensor-parallel rank's
    shard of every layer (cut on the host, so the device never holds more)."""
    cfg = cfg or config_from_hf(path)
    l0, l1 = layers or (0, cfg.layers)
    if not 0 <= l0 < l1 <= cfg.layers:
        raise ValueError(f"layer range [{l0}, {l1}) outside [0, {cfg.layers})")
    sh = _Shards(path)
    dev = torch.device(device)

    def get(name):
        return sh.get(name).to(dtype)

    def put(t):
        return t.contiguous().to(dev)

    shard = None
    if tp is not None and tp[1] > 1:
        from connex_b200.parallel.tp import shard_layer, tp_config
        shard = (lambda lw: shard_layer(lw, cfg, tp[0], tp[1]))
    out_layers = []
    for i in range(l0, l1):
        p = f"model.layers.{i}."
        q, k, v = get(p + "self_attn.q_proj.weight"), get(p + "self_attn.k_proj.weight"), \
            get(p + "self_attn.v_proj.weight")
        if q.shape != (cfg.heads * HEAD_DIM, cfg.hidden) or k.shape != (cfg.kv_heads * HEAD_DIM, cfg.hidden):
            raise ValueError(f"layer {i}: q/k shapes {tuple(q.shape)} / {tuple(k.shape)} do not match the config")
        lw = LayerWeights(
            attn_norm=get(p + "input_layernorm.weight"), wqkv=torch.cat([q, k, v], 0),
            wo=get(p + "self_attn.o_proj.weight"), mlp_norm=get(p + "post_attention_layernorm.weight"),
            w13=ops.interleave_gate_up(get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")),
            w2=get(p + "mlp.down_proj.weight"))
        if shard is not None:           # cut on the host: the device only ever holds this rank's part
            lw = shard(lw)
        out_layers.append(LayerWeights(**{name: put(t) for name, t in lw.__dict__.items()}))
    first, last = l0 == 0, l1 == cfg.layers
    embed = put(get("model.embed_tokens.weight")) if first else None
    head = None
    if last:
        if sh.has("lm_head.weight") and not _tied(path):
            head = put(get("lm_head.weight"))
        else:
            head = embed if embed is not None else put(get("model.embed_tokens.weight"))
    return LlamaWeights(cfg=tp_config(cfg, tp[1]) if shard is not None else cfg, embed=embed, layers=out_layers,
                        final_norm=put(get("model.norm.weight")) if last else None, lm_head=head)


def hf_config(cfg: LlamaConfig, tie: bool = False) -> dict:
    """The ``config.json`` of ``cfg`` (``LlamaForCausalLM``)."""
    c = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": cfg.vocab_size,
         "hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.heads,
         "num_key_value_heads": cfg.kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn,
         "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.eps, "max_position_embeddings": cfg.max_pos,
         "hidden_act": "silu", "tie_word_embeddings": tie, "torch_dtype": "bfloat16"}
    if cfg.rope_scaling is not None:
        f, lo, hi, orig = cfg.rope_scaling
        c["rope_scaling"] = {"rope_type": "llama3", "factor": f, "low_freq_factor": lo, "high_freq_factor": hi,
                             "original_max_position_embeddings": orig}
    return c


def hf_tensors(w: LlamaWeights) -> Iterable[Tuple[str, torch.Tensor]]:
    """(name, tensor) of ``w`` unfused into checkpoint names (host copies)."""
    cfg = w.cfg
    yield "model.embed_tokens.weight", w.embed
    for i, lw in enumerate(w.layers):
        p = f"model.layers.{i}."
        nq, nk = cfg.heads * HEAD_DIM, cfg.kv_heads * HEAD_DIM
        yield p + "input_layernorm.weight", lw.attn_norm
        yield p + "self_attn.q_proj.weight", lw.wqkv[:nq]
        yield p + "self_attn.k_proj.weight", lw.wqkv[nq:nq + nk]
        yield p + "self_attn.v_proj.weight", lw.wqkv[nq + nk:]
        yield p + "self_attn.o_proj.weight", lw.wo
        yield p + "post_attention_layernorm.weight", lw.mlp_norm
        gate, up = ops.deinterleave_gate_up(lw.w13)
        yield p + "mlp.gate_proj.weight", gate
        yield p + "mlp.up_proj.weight", up
        yield p + "mlp.down_proj.weight", lw.w2
    yield "model.norm.weight", w.final_norm
    yield "lm_head.weight", w.lm_head


def save_llama(w: LlamaWeights, path: str, max_shard_bytes: int = 4 << 30) -> None:
    """Write ``w`` as an HF checkpoint (``config.json`` + safetensors shards
    + ``model.safetensors.index.json``) that :func:`load_llama` and
    ``LlamaForCausalLM.from_pretrained`` read."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config(w.cfg), f, indent=1)
    shards, cur, size = [], {}, 0
    for name, t in hf_tensors(w):
        t = t.detach().to("cpu").contiguous()
        if cur and size + t.numel() * t.element_size() > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[name] = t
        size += t.numel() * t.element_size()
    shards.append(cur)
    index = {"metadata": {"total_size": 0}, "weight_map": {}}
    for n, sh in enumerate(shards):
        fname = f"model-{n + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, fname), metadata={"format": "pt"})
        for name, t in sh.items():
            index["weight_map"][name] = fname
            index["metadata"]["total_size"] += t.numel() * t.element_size()
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f, indent=1)
