"""Hugging Face Llama checkpoints (``config.json`` + ``*.safetensors``) onto
this engine's tensor-parallel shards.

The reference serves real checkpoints through sglang's loader
(docs/performance.md:3-5); this is the B200 build's equivalent for the
Llama family, so the engine and the HTTP server can run actual weights
instead of random ones.

A safetensors file is a little-endian u64 header length, a JSON header
``{name: {"dtype", "shape", "data_offsets"}, "__metadata__": ...}`` and the
raw tensor bytes. ``SafeTensors`` maps the file with numpy and slices rows or
columns before converting, so a rank reads only its shard of each tensor.
``write_safetensors`` writes the same format (tests, exports).
"""
import glob
import json
import os
import struct

import numpy as np
import torch

from .config import LlamaConfig

_DT = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16), "F32": (np.float32, torch.float32)}
_DT_NAME = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32"}


class SafeTensors:
    """Read-only view of one .safetensors file."""

    def __init__(self, path: str):
        self.path = path
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        self.meta = header.pop("__metadata__", {})
        self.entries = header
        self.data_start = 8 + n
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")

    def keys(self):
        return list(self.entries)

    def get(self, name: str, rows=None, cols=None) -> torch.Tensor:
        """Tensor ``name`` (CPU, stored dtype); ``rows`` / ``cols`` = (start,
        stop) of the first / second dimension."""
        e = self.entries[name]
        if e["dtype"] not in _DT:
            raise ValueError(f"{self.path}: {name} has unsupported dtype {e['dtype']}")
        np_dt, t_dt = _DT[e["dtype"]]
        a, b = e["data_offsets"]
        arr = self._mm[self.data_start + a:self.data_start + b].view(np_dt).reshape(e["shape"])
        if rows is not None:
            arr = arr[rows[0]:rows[1]]
        if cols is not None:
            arr = arr[:, cols[0]:cols[1]]
        t = torch.from_numpy(np.array(arr, copy=True))  # detach from the read-only map
        return t.view(t_dt) if e["dtype"] == "BF16" else t


def write_safetensors(path: str, tensors: dict, metadata: dict = None):
    """Write ``{name: tensor}`` (bf16 / fp16 / fp32, CPU or GPU) as safetensors."""
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        header[name] = {"dtype": _DT_NAME[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hdr = json.dumps(header).encode()
    hdr += b" " * (-len(hdr) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for raw in blobs:
            f.write(raw)


SUPPORTED_ARCHS = ("LlamaForCausalLM", "Qwen3ForCausalLM")


def config_from_hf(d: dict, name: str = None) -> LlamaConfig:
    """LlamaConfig from a Hugging Face ``config.json`` dict: LlamaForCausalLM,
    or Qwen3ForCausalLM (the same decoder plus per-head q/k RMSNorm)."""
    arch = (d.get("architectures") or ["LlamaForCausalLM"])[0]
    if arch not in SUPPORTED_ARCHS:
        raise ValueError(f"unsupported architecture {arch} (supported: {', '.join(SUPPORTED_ARCHS)})")
    if d.get("attention_bias") or d.get("mlp_bias"):
        raise ValueError("projection biases are not supported")
    heads = int(d["num_attention_heads"])
    hidden = int(d["hidden_size"])
    scaling = d.get("rope_scaling") or {}
    return LlamaConfig(
        name=name or d.get("_name_or_path") or d.get("model_type", "llama"),
        hidden=hidden, layers=int(d["num_hidden_layers"]), heads=heads,
        kv_heads=int(d.get("num_key_value_heads", heads)),
        head_dim=int(d.get("head_dim") or hidden // heads), ffn=int(d["intermediate_size"]),
        vocab=int(d["vocab_size"]), rope_theta=float(d.get("rope_theta", 10000.0)),
        eps=float(d.get("rms_norm_eps", 1e-5)), max_pos=int(d.get("max_position_embeddings", 8192)),
        rope_scaling=tuple(sorted((str(k), v) for k, v in scaling.items())),
        qk_norm=arch == "Qwen3ForCausalLM",
    )


class _Checkpoint:
    def __init__(self, model_dir: str):
        files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {model_dir}")
        self.files = [SafeTensors(f) for f in files]
        self.where = {k: f for f in self.files for k in f.keys()}

    def fetch(self, name, rows=None, cols=None):
        if name == "lm_head.weight" and name not in self.where:
            name = "model.embed_tokens.weight"  # tied embeddings
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name}")
        return self.where[name].get(name, rows, cols)


def load_llama(model_dir: str, tp_rank: int = 0, tp_size: int = 1, device="cuda"):
    """(LlamaConfig, LlamaWeights) of this TP rank from a Hugging Face Llama
    directory. Head dim 128 (the attention kernels' width) is required."""
    from .llama import _shard_weights

    with open(os.path.join(model_dir, "config.json")) as f:
        cfg = config_from_hf(json.load(f), name=os.path.basename(os.path.normpath(model_dir)))
    if cfg.head_dim != 128:
        raise ValueError(f"{model_dir}: head_dim {cfg.head_dim}; the attention kernels need 128")
    ck = _Checkpoint(model_dir)
    return cfg, _shard_weights(cfg, tp_rank, tp_size, device, ck.fetch)


def stop_token_ids(model_dir: str) -> tuple:
    """End-of-sequence token ids of a checkpoint: ``eos_token_id`` (an int or a
    list) from generation_config.json, else from config.json; () if none."""
    for name in ("generation_config.json", "config.json"):
        path = os.path.join(model_dir, name)
        if os.path.isfile(path):
            with open(path) as f:
                eos = json.load(f).get("eos_token_id")
            if eos is not None:
                return tuple(int(e) for e in (eos if isinstance(eos, list) else [eos]))
    return ()
