"""Hugging Face checkpoints of the Llama decoder family (Llama, Mistral,
Qwen2, Qwen3: ``config.json`` + ``*.safetensors``) onto this engine's
tensor-parallel shards.

The reference serves real checkpoints through sglang's loader
(docs/performance.md:3-5); this is the B200 build's equivalent for the
Llama family, so the engine and the HTTP server can run actual weights
instead of random ones.

A safetensors file is a little-endian u64 header length, a JSON header
``{name: {"dtype", "shape", "data_offsets"}, "__metadata__": ...}`` and the
raw tensor bytes. ``SafeTensors`` maps the file with numpy and slices rows or
columns before converting, so a rank reads only its shard of each tensor.
``write_safetensors`` writes the same format (tests, exports).

AWQ int4 checkpoints (the reference's served model is one: Qwen3.8-27B-AWQ,
docs/performance.md:3-5) load too: each quantized linear is dequantized to
bf16 as its TP shard is read, on the target device, and then runs on the
same bf16 tensor-core GEMMs as any other checkpoint (a 27B model is 54 GB in
bf16, well inside one B200's HBM).
"""
import glob
import json
import os
import struct

import numpy as np
import torch

from .config import LlamaConfig

_DT = {"BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16), "F32": (np.float32, torch.float32),
       "I32": (np.int32, torch.int32)}
_DT_NAME = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int32: "I32"}


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


SUPPORTED_ARCHS = ("LlamaForCausalLM", "Qwen3ForCausalLM", "Qwen2ForCausalLM", "MistralForCausalLM")


def config_from_hf(d: dict, name: str = None) -> LlamaConfig:
    """LlamaConfig from a Hugging Face ``config.json`` dict. Supported: the
    Llama decoder (LlamaForCausalLM, MistralForCausalLM), Qwen3ForCausalLM
    (plus per-head q/k RMSNorm) and Qwen2ForCausalLM (plus q/k/v biases).

    A sliding attention window (Mistral's ``sliding_window``, Qwen2's with
    ``use_sliding_window``) caps the positions at the window: every sequence
    the engine admits then fits inside it, where sliding and full attention
    are the same."""
    arch = (d.get("architectures") or ["LlamaForCausalLM"])[0]
    if arch not in SUPPORTED_ARCHS:
        raise ValueError(f"unsupported architecture {arch} (supported: {', '.join(SUPPORTED_ARCHS)})")
    if d.get("mlp_bias") or (d.get("attention_bias") and arch != "Qwen2ForCausalLM"):
        raise ValueError("projection biases are not supported (only Qwen2's q/k/v biases)")
    act = d.get("hidden_act", "silu")
    if act != "silu":  # the MLP kernel is SiLU(gate) * up
        raise ValueError(f"activation {act!r} is not supported (supported: silu)")
    heads = int(d["num_attention_heads"])
    hidden = int(d["hidden_size"])
    scaling = d.get("rope_scaling") or {}
    from ..ops import ROPE_SCALINGS

    kind = scaling.get("rope_type", scaling.get("type")) if scaling else None
    if kind not in ROPE_SCALINGS:
        raise ValueError(f"rope scaling {kind!r} is not supported (supported: linear, llama3)")
    max_pos = int(d.get("max_position_embeddings", 8192))
    window = None
    if arch == "MistralForCausalLM" or d.get("use_sliding_window"):
        window = d.get("sliding_window")
    if window:
        max_pos = min(max_pos, int(window))
    return LlamaConfig(
        name=name or d.get("_name_or_path") or d.get("model_type", "llama"),
        hidden=hidden, layers=int(d["num_hidden_layers"]), heads=heads,
        kv_heads=int(d.get("num_key_value_heads", heads)),
        head_dim=int(d.get("head_dim") or hidden // heads), ffn=int(d["intermediate_size"]),
        vocab=int(d["vocab_size"]), rope_theta=float(d.get("rope_theta", 10000.0)),
        eps=float(d.get("rms_norm_eps", 1e-5)), max_pos=max_pos,
        rope_scaling=tuple(sorted((str(k), v) for k, v in scaling.items())),
        qk_norm=arch == "Qwen3ForCausalLM",
        qkv_bias=arch == "Qwen2ForCausalLM",
    )


def config_to_hf(cfg: LlamaConfig) -> dict:
    """The Hugging Face ``config.json`` of a LlamaConfig (inverse of
    ``config_from_hf``)."""
    arch = "Qwen3ForCausalLM" if cfg.qk_norm else "Qwen2ForCausalLM" if cfg.qkv_bias else "LlamaForCausalLM"
    d = {"architectures": [arch], "model_type": arch[:-len("ForCausalLM")].lower(), "hidden_size": cfg.hidden,
         "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.heads, "num_key_value_heads": cfg.kv_heads,
         "head_dim": cfg.head_dim, "intermediate_size": cfg.ffn, "vocab_size": cfg.vocab,
         "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.eps, "max_position_embeddings": cfg.max_pos,
         "hidden_act": "silu", "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    if cfg.rope_scaling:
        d["rope_scaling"] = dict(cfg.rope_scaling)
    return d


def save_llama(model_dir: str, cfg: LlamaConfig, weights, shard_bytes: int = 4 << 30):
    """Write TP-1 bf16 ``weights`` as a Hugging Face checkpoint: config.json
    and safetensors files of at most ``shard_bytes`` each, fused qkv /
    gate_up split back into their projections. ``load_llama`` reads it back
    at any TP degree."""
    from ..ops import Int4Weight

    if weights.vocab_start != 0 or weights.embed.shape[0] != cfg.vocab:
        raise ValueError("save_llama needs the whole (TP-1) model")
    os.makedirs(model_dir, exist_ok=True)
    D = cfg.head_dim
    nq, nkv = cfg.heads * D, cfg.kv_heads * D
    t = {"model.embed_tokens.weight": weights.embed, "model.norm.weight": weights.norm,
         "lm_head.weight": weights.lm_head}
    for i, L in enumerate(weights.layers):
        if any(isinstance(v, Int4Weight) for v in L.values()):
            raise ValueError("save_llama writes bf16 weights (int4 layers found)")
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = L["ln1"]
        t[p + "post_attention_layernorm.weight"] = L["ln2"]
        q, k, v = L["qkv"][:nq], L["qkv"][nq:nq + nkv], L["qkv"][nq + nkv:]
        t[p + "self_attn.q_proj.weight"], t[p + "self_attn.k_proj.weight"], t[p + "self_attn.v_proj.weight"] = q, k, v
        t[p + "self_attn.o_proj.weight"] = L["o"]
        F_ = cfg.ffn
        t[p + "mlp.gate_proj.weight"], t[p + "mlp.up_proj.weight"] = L["gate_up"][:F_], L["gate_up"][F_:]
        t[p + "mlp.down_proj.weight"] = L["down"]
        if cfg.qk_norm:
            t[p + "self_attn.q_norm.weight"], t[p + "self_attn.k_norm.weight"] = L["q_norm"], L["k_norm"]
        if cfg.qkv_bias:
            b = L["qkv_bias"]
            t[p + "self_attn.q_proj.bias"], t[p + "self_attn.k_proj.bias"] = b[:nq], b[nq:nq + nkv]
            t[p + "self_attn.v_proj.bias"] = b[nq + nkv:]
    shards, cur, size = [], {}, 0
    for name, ten in t.items():
        nb = ten.numel() * ten.element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[name] = ten
        size += nb
    shards.append(cur)
    index = {}
    for j, sh in enumerate(shards):
        fname = f"model-{j + 1:05d}-of-{len(shards):05d}.safetensors"
        write_safetensors(os.path.join(model_dir, fname), sh, {"format": "pt"})
        index.update({k: fname for k in sh})
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(config_to_hf(cfg), f, indent=2)
    with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": index}, f, indent=2)


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


# AWQ "gemm" packing (AutoAWQ's format, which Hugging Face's AwqConfig reads):
# for a linear with K inputs and N outputs, ``qweight`` is int32 [K, N/8],
# ``qzeros`` int32 [K/G, N/8] and ``scales`` fp16 [K/G, N] for group size G.
# Bits 4i..4i+3 of a packed word hold output column 8c + _AWQ_ORDER[i], and
# W[k, n] = (q[k, n] - z[k // G, n]) * s[k // G, n].
_AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def awq_unpack(packed: torch.Tensor) -> torch.Tensor:
    """int32 [R, C] packed in AWQ order -> int32 [R, 8C] values 0..15, columns
    in natural order."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=packed.device)
    nib = (packed.unsqueeze(-1) >> shifts) & 0xF     # nib[..., i] = bits 4i..4i+3
    out = torch.empty_like(nib)
    out[..., list(_AWQ_ORDER)] = nib                  # column _AWQ_ORDER[i] <- nibble i
    return out.reshape(packed.shape[0], -1)


def awq_pack(q: torch.Tensor) -> torch.Tensor:
    """Inverse of ``awq_unpack``: values 0..15 [R, 8C] -> int32 [R, C]."""
    R, N = q.shape
    q = q.to(torch.int64).reshape(R, N // 8, 8)
    packed = torch.zeros(R, N // 8, dtype=torch.int64, device=q.device)
    for i, col in enumerate(_AWQ_ORDER):
        packed |= q[..., col] << (4 * i)
    return torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)


def awq_dequant(qweight, qzeros, scales, group: int) -> torch.Tensor:
    """fp32 [N, K] (Hugging Face [out, in] layout) from AWQ tensors."""
    q = awq_unpack(qweight)
    z = awq_unpack(qzeros).repeat_interleave(group, 0)
    s = scales.float().repeat_interleave(group, 0)
    return ((q - z).float() * s).t()


def awq_quantize(w: torch.Tensor, group: int = 128):
    """Round-to-nearest asymmetric int4 of an [N, K] weight in AWQ layout:
    (qweight, qzeros, scales fp16). Used to write AWQ-format test checkpoints;
    it does not search activation-aware scales."""
    wt = w.float().t()                                   # [K, N]
    K, N = wt.shape
    g = wt.reshape(K // group, group, N)
    lo, hi = g.amin(1), g.amax(1)
    s = ((hi - lo) / 15).clamp_min(1e-6).half()          # fp16, like the checkpoints
    sf = s.float()
    z = torch.round(-lo / sf).clamp(0, 15)
    q = torch.round(g / sf.unsqueeze(1) + z.unsqueeze(1)).clamp(0, 15).reshape(K, N)
    return awq_pack(q.to(torch.int32)), awq_pack(z.to(torch.int32)), s


def quantize_weights_int4(weights, group: int = 128):
    """Pack every decoder linear of ``weights`` (a LlamaWeights of any TP
    shard, on any device) as AWQ int4 in place (round-to-nearest per group),
    giving ``ops.Int4Weight`` linears: the int4 path measured on random
    weights. Returns ``weights``."""
    from ..ops import Int4Weight

    for L in weights.layers:
        for k in ("qkv", "o", "gate_up", "down"):
            qw, qz, s = awq_quantize(L[k], group)
            L[k] = Int4Weight(qw, qz, s, group)
    return weights


def awq_group_size(qc: dict) -> int:
    """Group size of a ``quantization_config`` this loader accepts (AWQ,
    4-bit, zero point, gemm packing); -1 = one group per input row range."""
    method = str(qc.get("quant_method", "")).lower()
    if method != "awq":
        raise ValueError(f"unsupported quantization {method or qc} (supported: awq)")
    if int(qc.get("bits", qc.get("w_bit", 4))) != 4 or not qc.get("zero_point", True):
        raise ValueError("AWQ checkpoints must be 4-bit with zero points")
    if str(qc.get("version", "gemm")).lower() != "gemm":
        raise ValueError(f"AWQ packing {qc.get('version')} is not supported (supported: gemm)")
    return int(qc.get("group_size", qc.get("q_group_size", 128)))


class _AwqCheckpoint(_Checkpoint):
    """A checkpoint whose linears may be AWQ-quantized: ``fetch`` of
    ``<prefix>.weight`` returns that shard dequantized when only
    ``<prefix>.qweight`` / ``qzeros`` / ``scales`` are stored. Unquantized
    modules (embeddings, norms, ``modules_to_not_convert``) read as usual."""

    def __init__(self, model_dir: str, group: int, device):
        super().__init__(model_dir)
        self.group = group
        self.device = torch.device(device)

    def _quantized(self, name):
        base = name[:-len(".weight")] if name.endswith(".weight") else None
        if base is None or name in self.where or base + ".qweight" not in self.where:
            return None
        return base

    def fetch(self, name, rows=None, cols=None):
        if self._quantized(name) is None:
            return super().fetch(name, rows, cols)
        qw, qz, sc, G = self._parts(name, rows, cols)
        return awq_dequant(qw, qz, sc, G)

    def fetch_int4(self, name, rows=None, cols=None):
        """The shard kept packed, as an ``ops.Int4Weight`` on the device
        (None for a module stored unquantized)."""
        from ..ops import Int4Weight

        if self._quantized(name) is None:
            return None
        qw, qz, sc, G = self._parts(name, rows, cols)
        return Int4Weight(qw.contiguous(), qz.contiguous(), sc.to(torch.float16).contiguous(), G)

    def _parts(self, name, rows=None, cols=None):
        """(qweight, qzeros, scales, group) of a shard, on the device."""
        base = self._quantized(name)
        qw = self.where[base + ".qweight"]
        K = qw.entries[base + ".qweight"]["shape"][0]
        G = K if self.group <= 0 else self.group
        # HF rows are output columns of the packed tensors; HF cols are their input rows
        out_cols = pk_cols = None
        if rows is not None:
            if rows[0] % 8 or rows[1] % 8:
                raise ValueError(f"{name}: output shard {rows} is not a multiple of 8 (AWQ packing)")
            out_cols, pk_cols = rows, (rows[0] // 8, rows[1] // 8)
        in_rows = grp_rows = None
        if cols is not None:
            if cols[0] % G or cols[1] % G:
                raise ValueError(f"{name}: input shard {cols} is not a multiple of the AWQ group {G}")
            in_rows, grp_rows = cols, (cols[0] // G, cols[1] // G)

        def part(suffix, r, c):
            return self.where[base + suffix].get(base + suffix, r, c).to(self.device)

        return (part(".qweight", in_rows, pk_cols), part(".qzeros", grp_rows, pk_cols),
                part(".scales", grp_rows, out_cols), G)


def load_llama(model_dir: str, tp_rank: int = 0, tp_size: int = 1, device="cuda", int4: bool = False):
    """(LlamaConfig, LlamaWeights) of this TP rank from a Hugging Face Llama
    directory (bf16 / fp16 / fp32, or AWQ int4: dequantized to bf16, or with
    ``int4`` kept packed as ``ops.Int4Weight`` for the int4 GEMV / dequant
    path). Head dim 128 (the attention kernels' width) is required."""
    from .llama import _shard_weights

    with open(os.path.join(model_dir, "config.json")) as f:
        hf = json.load(f)
    cfg = config_from_hf(hf, name=os.path.basename(os.path.normpath(model_dir)))
    if cfg.head_dim != 128:
        raise ValueError(f"{model_dir}: head_dim {cfg.head_dim}; the attention kernels need 128")
    qc = hf.get("quantization_config")
    ck = _AwqCheckpoint(model_dir, awq_group_size(qc), device) if qc else _Checkpoint(model_dir)
    linear = ck.fetch_int4 if (int4 and qc) else None
    return cfg, _shard_weights(cfg, tp_rank, tp_size, device, ck.fetch, linear)


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
