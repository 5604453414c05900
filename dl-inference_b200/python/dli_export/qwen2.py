"""Qwen2 lowering to dli.graph.v1 for the sm_100a plugin.

Extends the reference exporter's Qwen2 lowering (python/dli_export/export.py:
250-457 of yncxcw/dl-inference), which is batch-1, single-token, MHA-only and
fp32, to what the plugin serves:

* GQA (any num_key_value_heads dividing num_attention_heads; the reference
  rejects GQA at export.py:256-260);
* [B, S] token batches with a per-sequence `positions` input (int64 [B], the
  cache row of each sequence's first token), so one graph serves prefill and
  every decode step (the reference bakes start_pos at 0, export.py:350-356);
* a preallocated KV cache addressed by position (fused `qkv_rotary_cache`
  writes rotated k and v into the rows, `attention_kvcache` reads them);
* fused QKV and gate/up projections, `add_rms_norm` for residual + norm,
  `silu_mul` for SwiGLU, and an LM head over the last token only;
* bf16/fp16 weights (the reference casts every weight to fp32, weights.py:39-40);
* q/k row permutation inside each head so the reference's interleaved-pair
  rotary (rotary/kernel.py:22-35) equals the source model's rotate-half RoPE;
* Megatron tensor parallelism: q/k/v and gate/up split by heads/columns,
  o_proj/down_proj split by input columns, an `all_reduce` after each.

The weight transform works on any torch tensors (CPU or CUDA), so large
synthetic models can be built directly on the GPU.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, asdict
from pathlib import Path
from typing import Any

import torch


@dataclass(frozen=True)
class Qwen2Shape:
    hidden: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_embeddings: bool = False

    @staticmethod
    def from_hf(config: Any) -> "Qwen2Shape":
        heads = int(config.num_attention_heads)
        hidden = int(config.hidden_size)
        head_dim = int(getattr(config, "head_dim", None) or hidden // heads)
        theta = getattr(config, "rope_theta", None)
        if theta is None:
            rp = getattr(config, "rope_parameters", None) or {}
            theta = rp.get("rope_theta", 10000.0)
        return Qwen2Shape(hidden=hidden, layers=int(config.num_hidden_layers), q_heads=heads,
                          kv_heads=int(config.num_key_value_heads), head_dim=head_dim,
                          intermediate=int(config.intermediate_size), vocab=int(config.vocab_size),
                          rms_eps=float(config.rms_norm_eps), rope_theta=float(theta),
                          tie_embeddings=bool(getattr(config, "tie_word_embeddings", False)))

    def params(self) -> int:
        attn = self.hidden * (self.q_heads + 2 * self.kv_heads) * self.head_dim \
            + (self.q_heads + 2 * self.kv_heads) * self.head_dim \
            + self.q_heads * self.head_dim * self.hidden
        mlp = 3 * self.hidden * self.intermediate
        body = self.layers * (attn + mlp + 2 * self.hidden) + self.hidden
        emb = self.vocab * self.hidden
        return body + emb + (0 if self.tie_embeddings else emb)


# Shapes named by the benchmark configs.
QWEN2_0_5B = Qwen2Shape(896, 24, 14, 2, 64, 4864, 151936, tie_embeddings=True)
QWEN2_7B = Qwen2Shape(3584, 28, 28, 4, 128, 18944, 152064)
QWEN2_72B = Qwen2Shape(8192, 80, 64, 8, 128, 29568, 152064)


def rotary_tables(shape: Qwen2Shape, max_positions: int) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [max_positions, head_dim/2] fp32 with inv_freq_i = theta^(-2i/D),
    as the reference exporter builds them (export.py:228-247)."""
    d = shape.head_dim
    inv = 1.0 / (shape.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    freqs = torch.outer(torch.arange(max_positions, dtype=torch.float64), inv)
    return torch.cos(freqs).float().contiguous(), torch.sin(freqs).float().contiguous()


def interleave_permutation(head_dim: int) -> torch.Tensor:
    """Row order [0, D/2, 1, D/2+1, ...]: interleaved pair i of the permuted head
    holds dims (i, i + D/2) of the original head, so rotating interleaved pairs
    applies the rotate-half rotation with frequency i."""
    half = head_dim // 2
    return torch.stack([torch.arange(half), torch.arange(half) + half], dim=1).reshape(-1)


def _permute_heads(t: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    perm = interleave_permutation(head_dim).to(t.device)
    shp = t.shape
    x = t.reshape(heads, head_dim, *shp[1:])
    return x.index_select(1, perm).reshape(shp)


GLU_BLOCK = 64


def vocab_parallel(shape: "Qwen2Shape", tp_size: int) -> bool:
    """With tensor parallelism the LM head is split by vocabulary rows (each rank
    streams V/tp rows per token and a tp_argmax node picks the global id), when
    the vocabulary divides evenly; otherwise it is replicated."""
    return tp_size > 1 and shape.vocab % tp_size == 0


def glu_blocked(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[I, K] gate and up weights -> the layout of the fused `linear_silu_mul`
    operator: 64-row blocks, rows [128b, 128b+64) = gate rows [64b, 64b+64) and
    rows [128b+64, 128b+128) = the matching up rows; rows past I are zero. One
    128-row tensor-core tile then holds matching gate and up rows."""
    inter, k = w_gate.shape
    blocks = (inter + GLU_BLOCK - 1) // GLU_BLOCK
    g = torch.zeros(blocks * GLU_BLOCK, k, dtype=w_gate.dtype, device=w_gate.device)
    u = torch.zeros_like(g)
    g[:inter], u[:inter] = w_gate, w_up
    return torch.stack([g.view(blocks, GLU_BLOCK, k), u.view(blocks, GLU_BLOCK, k)], 1) \
        .reshape(2 * blocks * GLU_BLOCK, k).contiguous()


def glu_unblocked(w_glu: torch.Tensor, inter: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of glu_blocked: (gate [I, K], up [I, K])."""
    k = w_glu.shape[-1]
    b = w_glu.reshape(-1, 2, GLU_BLOCK, k)
    return b[:, 0].reshape(-1, k)[:inter], b[:, 1].reshape(-1, k)[:inter]


def transform_weights(state: dict[str, torch.Tensor], shape: Qwen2Shape, tp_size: int = 1,
                      tp_rank: int = 0, dtype: torch.dtype | None = None,
                      layers: range | None = None, fused_glu: bool = True) -> dict[str, torch.Tensor]:
    """HF-named Qwen2 state dict -> plugin weights for one tensor-parallel rank.

    Output names: embed, layers.{i}.{ln_in,wqkv,bqkv,wo,ln_post,wgu,wd}, norm,
    lm_head. Tensors are contiguous and cast to `dtype` when given. `wgu` is
    [gate; up] for the linear + silu_mul graph, or the glu_blocked() layout of
    the fused linear_silu_mul operator when `fused_glu`.
    """
    hq, hkv, d, inter = shape.q_heads, shape.kv_heads, shape.head_dim, shape.intermediate
    if hq % tp_size or hkv % tp_size or inter % tp_size:
        raise ValueError(f"tp_size {tp_size} must divide heads ({hq}/{hkv}) and intermediate ({inter})")
    qh, kh, ish = hq // tp_size, hkv // tp_size, inter // tp_size
    cast = (lambda t: t.to(dtype).contiguous()) if dtype is not None else (lambda t: t.contiguous())
    out: dict[str, torch.Tensor] = {}
    full = "model.embed_tokens.weight" in state  # a per-layer slice carries no embeddings
    if full:
        out["embed"] = cast(state["model.embed_tokens.weight"])
    layers = layers if layers is not None else range(shape.layers)
    for i in layers:
        p = f"model.layers.{i}."
        q_w = _permute_heads(state[p + "self_attn.q_proj.weight"], hq, d)
        k_w = _permute_heads(state[p + "self_attn.k_proj.weight"], hkv, d)
        v_w = state[p + "self_attn.v_proj.weight"]
        q_b = _permute_heads(state[p + "self_attn.q_proj.bias"], hq, d)
        k_b = _permute_heads(state[p + "self_attn.k_proj.bias"], hkv, d)
        v_b = state[p + "self_attn.v_proj.bias"]
        qs = slice(tp_rank * qh * d, (tp_rank + 1) * qh * d)
        ks = slice(tp_rank * kh * d, (tp_rank + 1) * kh * d)
        out[f"layers.{i}.wqkv"] = cast(torch.cat([q_w[qs], k_w[ks], v_w[ks]], 0))
        out[f"layers.{i}.bqkv"] = cast(torch.cat([q_b[qs], k_b[ks], v_b[ks]], 0))
        out[f"layers.{i}.wo"] = cast(state[p + "self_attn.o_proj.weight"][:, qs])
        isl = slice(tp_rank * ish, (tp_rank + 1) * ish)
        gate, up = state[p + "mlp.gate_proj.weight"][isl], state[p + "mlp.up_proj.weight"][isl]
        out[f"layers.{i}.wgu"] = cast(glu_blocked(gate, up) if fused_glu else torch.cat([gate, up], 0))
        out[f"layers.{i}.wd"] = cast(state[p + "mlp.down_proj.weight"][:, isl])
        out[f"layers.{i}.ln_in"] = cast(state[p + "input_layernorm.weight"])
        out[f"layers.{i}.ln_post"] = cast(state[p + "post_attention_layernorm.weight"])
    if full:
        out["norm"] = cast(state["model.norm.weight"])
        lm = state.get("lm_head.weight")
        lm = lm if lm is not None else state["model.embed_tokens.weight"]
        if vocab_parallel(shape, tp_size):  # rank r holds ids [r*V/tp, (r+1)*V/tp)
            vs = shape.vocab // tp_size
            lm = lm[tp_rank * vs:(tp_rank + 1) * vs]
        out["lm_head"] = cast(lm)
    return out


def build_graph(shape: Qwen2Shape, capacity: int, tp_size: int = 1, model_type: str = "qwen2",
                weights_file: str = "", with_argmax: bool = True, fused_glu: bool = True,
                logits_dtype: str | None = "float32",
                residual_dtype: str | None = "float32", fused_exchange: bool = True,
                fused_qkv_rotary: bool = True) -> dict[str, Any]:
    """dli.graph.v1 dict for one rank. Inputs: input_ids [B,S] int64, positions [B]
    int64, rotary_cos/rotary_sin, and the weights of transform_weights() (made
    with the same `fused_glu`: one linear_silu_mul node instead of linear +
    silu_mul; the fused operator serves bfloat16/float16). `logits_dtype` sets
    the LM head's output type: "float32" keeps the fp32 accumulator, so greedy
    ids are not decided among logits that rounding to bf16 made equal; None
    writes the weights' dtype. `residual_dtype` = "float32" keeps the residual
    stream (embedding output + every block's output) in fp32: a cast after the
    embedding starts it and each add_rms_norm adds the block's bf16 output to it
    unrounded, so a 16-bit model does not round its running sum once per layer
    (None keeps the residual in the weights' dtype). With tensor parallelism,
    `fused_exchange` makes each row-split projection and the all-reduce + add +
    RMSNorm after it one `linear_all_reduce_add_rms_norm` node, whose decode
    GEMM pushes its partial rows into the group's exchange buffers itself.
    `fused_qkv_rotary` makes the q|k|v projection and its rotary + KV-cache
    write one `linear_qkv_rotary_cache` node (decode GEMMs rotate and scatter
    in their epilogue)."""
    hq, hkv, d = shape.q_heads // tp_size, shape.kv_heads // tp_size, shape.head_dim
    nodes: list[dict[str, Any]] = []

    def node(name, op, inputs, outputs, attrs=None):
        nodes.append({"name": name, "op": op, "inputs": inputs, "outputs": outputs, "attrs": attrs or {}})

    eps = float(shape.rms_eps)
    # residual add + RMSNorm after a row-split projection; with tensor parallelism
    # the projection's output is a partial sum, all-reduced by the same node
    add_norm = "all_reduce_add_rms_norm" if tp_size > 1 else "add_rms_norm"
    fuse = fused_exchange and tp_size > 1

    def project_add_norm(name, resid_in, x_in, w_in, ln, outs, proj_name, part):
        """row-split projection + (all-reduce) + residual add + RMSNorm"""
        if fuse:
            node(name, "linear_all_reduce_add_rms_norm", [resid_in, x_in, w_in, ln], outs, {"eps": eps})
        else:
            node(proj_name, "linear", [x_in, w_in], [part])
            node(name, add_norm, [resid_in, part, ln], outs, {"eps": eps})

    node("embed_tokens", "embedding", ["input_ids", "embed"], ["h0"])
    resid, pending = "h0", None  # pending: the previous layer's (down input, down weight, name)
    if residual_dtype:
        node("residual_stream", "cast", ["h0"], ["h0_res"], {"dtype": residual_dtype})
        resid = "h0_res"
    for i in range(shape.layers):
        L = f"layers.{i}"
        if pending is None:
            node(f"{L}.input_layernorm", "rms_norm", ["h0", f"{L}.ln_in"], [f"{L}.x"], {"eps": eps})
        else:
            project_add_norm(f"{L}.input_layernorm", resid, pending[0], pending[1], f"{L}.ln_in",
                             [f"{L}.x", f"{L}.h_in"], pending[2], pending[3])
            resid = f"{L}.h_in"
        rot_attrs = {"q_heads": hq, "kv_heads": hkv, "head_dim": d, "capacity": int(capacity),
                     "kv_cache": f"layer_{i}"}
        if fused_qkv_rotary:
            node(f"{L}.qkv_proj", "linear_qkv_rotary_cache",
                 [f"{L}.x", f"{L}.wqkv", f"{L}.bqkv", "rotary_cos", "rotary_sin", "positions"], [f"{L}.q"],
                 rot_attrs)
        else:
            node(f"{L}.qkv_proj", "linear", [f"{L}.x", f"{L}.wqkv", f"{L}.bqkv"], [f"{L}.qkv"])
            node(f"{L}.rotary_cache", "qkv_rotary_cache",
                 [f"{L}.qkv", "rotary_cos", "rotary_sin", "positions"], [f"{L}.q"], rot_attrs)
        node(f"{L}.attention", "attention_kvcache", [f"{L}.q", "positions"], [f"{L}.attn"],
             {"kv_cache": f"layer_{i}"})
        project_add_norm(f"{L}.post_attention_layernorm", resid, f"{L}.attn", f"{L}.wo", f"{L}.ln_post",
                         [f"{L}.x2", f"{L}.h_mid"], f"{L}.o_proj", f"{L}.o_part")
        resid = f"{L}.h_mid"
        if fused_glu:
            node(f"{L}.gate_up_proj", "linear_silu_mul", [f"{L}.x2", f"{L}.wgu"], [f"{L}.act"],
                 {"intermediate": shape.intermediate // tp_size})
        else:
            node(f"{L}.gate_up_proj", "linear", [f"{L}.x2", f"{L}.wgu"], [f"{L}.gu"])
            node(f"{L}.act", "silu_mul", [f"{L}.gu"], [f"{L}.act"])
        pending = (f"{L}.act", f"{L}.wd", f"{L}.down_proj", f"{L}.d_part")
    project_add_norm("norm", resid, pending[0], pending[1], "norm", ["normed", "h_out"], pending[2], pending[3])
    node("last_token", "last_token", ["normed"], ["last_hidden"])
    # with a vocab-parallel LM head, `logits` is this rank's slice of the vocabulary
    node("lm_head", "linear", ["last_hidden", "lm_head"], ["logits"],
         {"out_dtype": logits_dtype} if logits_dtype else None)
    outputs = ["logits"]
    if with_argmax:
        node("greedy", "tp_argmax" if vocab_parallel(shape, tp_size) else "argmax", ["logits"], ["next_ids"])
        outputs.append("next_ids")
    return {"format": "dli.graph.v1", "model_type": model_type, "weights": weights_file,
            "inputs": ["input_ids", "positions"], "outputs": outputs, "nodes": nodes}


def random_state(shape: Qwen2Shape, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 std: float = 0.02, layers: range | None = None,
                 embeddings: bool = True) -> dict[str, torch.Tensor]:
    """HF-named random weights: every matrix and bias ~ N(0, std), norm weights 1.0
    (the source model's initial value). `embeddings=False` leaves out the
    embedding, final norm and LM head (per-layer generation of large models)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def rn(*s):
        return (torch.randn(*s, device=device, generator=g, dtype=torch.float32) * std).to(dtype)

    hq, hkv, d, h, i_ = shape.q_heads, shape.kv_heads, shape.head_dim, shape.hidden, shape.intermediate
    st: dict[str, torch.Tensor] = {}
    if embeddings:
        st["model.embed_tokens.weight"] = rn(shape.vocab, h)
    for i in (layers if layers is not None else range(shape.layers)):
        p = f"model.layers.{i}."
        st[p + "self_attn.q_proj.weight"] = rn(hq * d, h)
        st[p + "self_attn.q_proj.bias"] = rn(hq * d)
        st[p + "self_attn.k_proj.weight"] = rn(hkv * d, h)
        st[p + "self_attn.k_proj.bias"] = rn(hkv * d)
        st[p + "self_attn.v_proj.weight"] = rn(hkv * d, h)
        st[p + "self_attn.v_proj.bias"] = rn(hkv * d)
        st[p + "self_attn.o_proj.weight"] = rn(h, hq * d)
        st[p + "mlp.gate_proj.weight"] = rn(i_, h)
        st[p + "mlp.up_proj.weight"] = rn(i_, h)
        st[p + "mlp.down_proj.weight"] = rn(h, i_)
        st[p + "input_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
        st[p + "post_attention_layernorm.weight"] = torch.ones(h, device=device, dtype=dtype)
    if embeddings:
        st["model.norm.weight"] = torch.ones(h, device=device, dtype=dtype)
        if not shape.tie_embeddings:
            st["lm_head.weight"] = rn(shape.vocab, h)
    return st


_DTYPE_NAMES = {torch.float32: "float32", torch.int64: "int64", torch.bfloat16: "bfloat16",
                torch.float16: "float16", torch.int32: "int32"}


def write_weights(tensors: dict[str, torch.Tensor], out_dir: Path, stem: str) -> Path:
    """dli.weights.v1 manifest + payload (python/dli_export/weights.py:52-65 format)."""
    out_dir.mkdir(parents=True, exist_ok=True)
    data_name = f"{stem}.dli.weights.bin"
    manifest: dict[str, Any] = {"format": "dli.weights.v1", "data": data_name, "tensors": {}}
    offset = 0
    with (out_dir / data_name).open("wb") as f:
        for name, t in tensors.items():
            host = t.detach().cpu().contiguous()
            payload = host.view(torch.uint8).numpy().tobytes() if host.numel() else b""
            f.write(payload)
            manifest["tensors"][name] = {"dtype": _DTYPE_NAMES[host.dtype], "shape": list(host.shape),
                                         "offset": offset, "nbytes": len(payload)}
            offset += len(payload)
    path = out_dir / f"{stem}.dli.weights.json"
    path.write_text(json.dumps(manifest, indent=1), encoding="utf-8")
    return path


def export_qwen2(model_or_state: Any, out_dir: str | Path, stem: str = "qwen2",
                 shape: Qwen2Shape | None = None, capacity: int = 4096, tp_size: int = 1,
                 tp_rank: int = 0, dtype: torch.dtype = torch.bfloat16) -> tuple[Path, Path]:
    """Writes <stem>.dli.json and <stem>.dli.weights.{json,bin} for one TP rank.
    `model_or_state` is an HF Qwen2ForCausalLM or its state dict."""
    out = Path(out_dir)
    if hasattr(model_or_state, "state_dict"):
        shape = shape or Qwen2Shape.from_hf(model_or_state.config)
        state = {k: v.detach() for k, v in model_or_state.state_dict().items()}
    else:
        state = model_or_state
    if shape is None:
        raise ValueError("shape is required with a state dict")
    fused = dtype in (torch.bfloat16, torch.float16)  # the fused SwiGLU GEMM is 16-bit only
    weights = transform_weights(state, shape, tp_size, tp_rank, dtype, fused_glu=fused)
    cos, sin = rotary_tables(shape, capacity)
    weights["rotary_cos"], weights["rotary_sin"] = cos, sin
    wpath = write_weights(weights, out, stem)
    graph = build_graph(shape, capacity, tp_size, weights_file=wpath.name, fused_glu=fused)
    gpath = out / f"{stem}.dli.json"
    gpath.write_text(json.dumps(graph, indent=1), encoding="utf-8")
    meta = {"shape": asdict(shape), "capacity": capacity, "tp_size": tp_size, "tp_rank": tp_rank}
    (out / f"{stem}.meta.json").write_text(json.dumps(meta, indent=1), encoding="utf-8")
    return gpath, wpath


def decode_bytes_per_step(shape: Qwen2Shape, batch: int, context: int) -> int:
    """Algorithmic HBM bytes of one decode step (bf16): every weight once (embedding
    rows excluded except the LM head) plus reading `context` cached tokens and
    writing one per sequence."""
    hq, hkv, d = shape.q_heads, shape.kv_heads, shape.head_dim
    body = shape.layers * (shape.hidden * (hq + 2 * hkv) * d + (hq + 2 * hkv) * d
                           + hq * d * shape.hidden + 3 * shape.hidden * shape.intermediate
                           + 2 * shape.hidden) + shape.hidden
    lm = shape.vocab * shape.hidden
    kv_per_token = 2 * shape.layers * hkv * d
    return 2 * (body + lm + batch * (context + 1) * kv_per_token)


def prefill_flops(shape: Qwen2Shape, batch: int, seq: int) -> float:
    """Algorithmic FLOPs of a causal prefill: 2 * body params * tokens + causal
    attention (QK^T and PV over the lower triangle) + last-token LM head."""
    hq, hkv, d = shape.q_heads, shape.kv_heads, shape.head_dim
    body = shape.layers * (shape.hidden * (hq + 2 * hkv) * d + hq * d * shape.hidden
                           + 3 * shape.hidden * shape.intermediate)
    attn = 2.0 * batch * shape.layers * hq * d * seq * (seq + 1)  # 2 GEMMs x 2 flop x S(S+1)/2
    return 2.0 * body * batch * seq + attn + 2.0 * shape.vocab * shape.hidden * batch


def param_count(shape: Qwen2Shape) -> int:
    return shape.params()


__all__ = ["Qwen2Shape", "QWEN2_0_5B", "QWEN2_7B", "QWEN2_72B", "rotary_tables", "transform_weights",
           "build_graph", "random_state", "write_weights", "export_qwen2", "interleave_permutation",
           "decode_bytes_per_step", "prefill_flops", "param_count"]

_ = math
