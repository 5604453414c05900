"""CPU tests of the Qwen2 lowering (dli_export.qwen2): graph structure, the q/k
row permutation that maps the reference's interleaved rotary onto the source
model's rotate-half RoPE, and tensor-parallel sharding."""
from __future__ import annotations

import json

import numpy as np
import torch

from dli_export.qwen2 import (Qwen2Shape, build_graph, export_qwen2, glu_unblocked, interleave_permutation,
                              random_state, rotary_tables, transform_weights)
from oracle import ops as O

TINY = Qwen2Shape(hidden=64, layers=2, q_heads=4, kv_heads=2, head_dim=16, intermediate=96, vocab=50)


def rotate_half_rope(x, cos, sin, pos):
    """Source-model RoPE on [.., S, D]: x*cos + rotate_half(x)*sin with cos/sin
    duplicated over both halves."""
    half = x.shape[-1] // 2
    c = np.concatenate([cos[pos], cos[pos]], -1)
    s = np.concatenate([sin[pos], sin[pos]], -1)
    rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
    return x * c + rot * s


def test_interleaved_rotary_on_permuted_rows_equals_rotate_half():
    rng = np.random.default_rng(0)
    d, s = 16, 5
    cos, sin = rotary_tables(TINY, 32)
    x = rng.standard_normal((1, 1, s, d))
    perm = interleave_permutation(d).numpy()
    xp = x[..., perm]
    rot_interleaved, _ = O.rotary(xp, xp, cos.numpy(), sin.numpy(), start_pos=3)
    ref = rotate_half_rope(x, cos.numpy().astype(np.float64), sin.numpy().astype(np.float64),
                           np.arange(3, 3 + s))
    np.testing.assert_allclose(rot_interleaved, ref[..., perm], rtol=1e-6, atol=1e-6)
    # attention scores are invariant to the shared permutation of q and k
    q = rng.standard_normal((1, 1, s, d))
    k = rng.standard_normal((1, 1, s, d))
    np.testing.assert_allclose(q[..., perm] @ k[..., perm].swapaxes(-1, -2), q @ k.swapaxes(-1, -2))


def test_graph_structure_per_layer():
    g = build_graph(TINY, capacity=64, tp_size=1, fused_glu=False, residual_dtype=None, fused_qkv_rotary=False)
    ops = [n["op"] for n in g["nodes"]]
    assert ops[0] == "embedding"
    layer0 = ["rms_norm", "linear", "qkv_rotary_cache", "attention_kvcache", "linear", "add_rms_norm",
              "linear", "silu_mul", "linear"]
    layer1 = ["add_rms_norm"] + layer0[1:]
    assert ops[1:1 + 9] == layer0
    assert ops[10:19] == layer1
    assert ops[19:] == ["add_rms_norm", "last_token", "linear", "argmax"]
    # fused SwiGLU: gate/up projection + silu_mul become one node
    gf = build_graph(TINY, capacity=64, tp_size=1)
    fused = [n for n in gf["nodes"] if n["op"] == "linear_silu_mul"]
    assert len(fused) == TINY.layers and "silu_mul" not in [n["op"] for n in gf["nodes"]]
    assert fused[0]["attrs"]["intermediate"] == TINY.intermediate
    # fp32 residual stream (default): a cast after the embedding starts it; the
    # first norm still reads the embedding output, every add+norm the fp32 chain
    cast = [n for n in gf["nodes"] if n["op"] == "cast"]
    assert len(cast) == 1 and cast[0]["inputs"] == ["h0"] and cast[0]["attrs"]["dtype"] == "float32"
    first_add = next(n for n in gf["nodes"] if n["op"] == "add_rms_norm")
    assert first_add["inputs"][0] == "h0_res"
    assert gf["nodes"][2]["op"] == "rms_norm" and gf["nodes"][2]["inputs"][0] == "h0"
    lm = next(n for n in gf["nodes"] if n["name"] == "lm_head")
    assert lm["attrs"]["out_dtype"] == "float32"
    assert g["inputs"] == ["input_ids", "positions"] and g["outputs"] == ["logits", "next_ids"]
    g2 = build_graph(TINY, capacity=64, tp_size=2, fused_exchange=False)
    ops2 = [n["op"] for n in g2["nodes"]]
    # every add_rms_norm after a row-split projection becomes the all-reduce form
    assert ops2.count("all_reduce_add_rms_norm") == 2 * TINY.layers
    assert "add_rms_norm" not in ops2 and "all_reduce" not in ops2
    assert ops2[-1] == "tp_argmax" and ops[-1] == "argmax"
    # fused (default): each row-split projection and the all-reduce + add + norm
    # after it are one node reading the projection's input and weight
    g3 = build_graph(TINY, capacity=64, tp_size=2)
    fx = [n for n in g3["nodes"] if n["op"] == "linear_all_reduce_add_rms_norm"]
    assert len(fx) == 2 * TINY.layers and "all_reduce_add_rms_norm" not in [n["op"] for n in g3["nodes"]]
    assert fx[0]["inputs"][1:3] == ["layers.0.attn", "layers.0.wo"]
    assert fx[1]["inputs"][1:3] == ["layers.0.act", "layers.0.wd"]
    assert fx[-1]["name"] == "norm" and fx[-1]["outputs"] == ["normed", "h_out"]
    assert len(g3["nodes"]) == len(g2["nodes"]) - 2 * TINY.layers
    rc = next(n for n in g2["nodes"] if n["op"] == "linear_qkv_rotary_cache")
    assert rc["attrs"]["q_heads"] == 2 and rc["attrs"]["kv_heads"] == 1
    # fused q|k|v projection + rotary + cache write (default): one node per layer
    qr = [n for n in gf["nodes"] if n["op"] == "linear_qkv_rotary_cache"]
    assert len(qr) == TINY.layers and "qkv_rotary_cache" not in [n["op"] for n in gf["nodes"]]
    assert qr[0]["inputs"] == ["layers.0.x", "layers.0.wqkv", "layers.0.bqkv", "rotary_cos", "rotary_sin",
                               "positions"] and qr[0]["outputs"] == ["layers.0.q"]


def test_tensor_parallel_shards_recompose():
    st = random_state(TINY, dtype=torch.float32, seed=3)
    full = transform_weights(st, TINY, 1, 0)
    shards = [transform_weights(st, TINY, 2, r) for r in range(2)]
    d, hq, hkv = TINY.head_dim, TINY.q_heads, TINY.kv_heads
    for i in range(TINY.layers):
        w = full[f"layers.{i}.wqkv"]
        q, k, v = w[:hq * d], w[hq * d:(hq + hkv) * d], w[(hq + hkv) * d:]
        parts = [s[f"layers.{i}.wqkv"] for s in shards]
        qh, kh = hq // 2 * d, hkv // 2 * d
        torch.testing.assert_close(torch.cat([p[:qh] for p in parts]), q)
        torch.testing.assert_close(torch.cat([p[qh:qh + kh] for p in parts]), k)
        torch.testing.assert_close(torch.cat([p[qh + kh:] for p in parts]), v)
        torch.testing.assert_close(torch.cat([s[f"layers.{i}.wo"] for s in shards], 1), full[f"layers.{i}.wo"])
        torch.testing.assert_close(torch.cat([s[f"layers.{i}.wd"] for s in shards], 1), full[f"layers.{i}.wd"])
        inter = TINY.intermediate
        p = f"model.layers.{i}.mlp."
        # fused layout: 64-row gate/up blocks, zero-padded (96 -> 128 rows, 48 -> 64 per shard)
        assert full[f"layers.{i}.wgu"].shape[0] == 2 * 128 and shards[0][f"layers.{i}.wgu"].shape[0] == 2 * 64
        g_full, u_full = glu_unblocked(full[f"layers.{i}.wgu"], inter)
        torch.testing.assert_close(g_full, st[p + "gate_proj.weight"])
        torch.testing.assert_close(u_full, st[p + "up_proj.weight"])
        gs = [glu_unblocked(s[f"layers.{i}.wgu"], inter // 2) for s in shards]
        torch.testing.assert_close(torch.cat([g for g, _ in gs]), g_full)
        torch.testing.assert_close(torch.cat([u for _, u in gs]), u_full)
        assert not full[f"layers.{i}.wgu"].reshape(2, 2, 64, -1)[1, :, 32:].any()  # padding rows
        # unfused layout: [gate; up]
        plain = transform_weights(st, TINY, 1, 0, fused_glu=False)[f"layers.{i}.wgu"]
        torch.testing.assert_close(plain, torch.cat([g_full, u_full]))


def test_export_writes_loadable_graph_and_weights(tmp_path):
    import dli

    st = random_state(TINY, dtype=torch.bfloat16, seed=1)
    gpath, wpath = export_qwen2(st, tmp_path, "tiny", shape=TINY, capacity=64)
    graph = dli.Graph.from_json_file(str(gpath))
    assert graph.inputs == ["input_ids", "positions"]
    assert graph.num_nodes == len(json.loads(gpath.read_text())["nodes"])
    weights = dli.load_weights(str(wpath), "cpu")
    ref = transform_weights(st, TINY, 1, 0, torch.bfloat16)
    for name, t in ref.items():
        assert torch.equal(weights[name], t), name
    assert weights["rotary_cos"].dtype == torch.float32 and weights["rotary_cos"].shape == (64, 8)


def _hf_tiny(shape):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(vocab_size=shape.vocab, hidden_size=shape.hidden,
                      intermediate_size=shape.intermediate, num_hidden_layers=shape.layers,
                      num_attention_heads=shape.q_heads, num_key_value_heads=shape.kv_heads,
                      max_position_embeddings=256, rms_norm_eps=shape.rms_eps,
                      rope_theta=shape.rope_theta, tie_word_embeddings=shape.tie_embeddings,
                      attn_implementation="eager")
    return Qwen2ForCausalLM(cfg).double().eval()


def test_exported_graph_on_the_oracle_matches_the_source_model():
    """The lowering (fused/permuted/sharded weights + graph) executed by the CPU
    oracle reproduces transformers' Qwen2 in float64, prefill and decode, at TP 1 and 2.
    Tolerance 1e-4 relative: both sides use fp32 rotary angle tables, computed in a
    different order; any structural error (weight order, head split, permutation)
    shows up at O(1)."""
    from oracle.graph import GraphOracle

    st = random_state(TINY, dtype=torch.float32, seed=5, std=0.2)
    hf = _hf_tiny(TINY)
    hf.load_state_dict({k: v.double() for k, v in st.items()}, strict=False)
    ids = torch.randint(0, TINY.vocab, (2, 6), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        ref_prefill = hf(ids).logits[:, -1].numpy()
        nxt = torch.tensor([[3], [7]])
        ref_decode = hf(torch.cat([ids, nxt], 1)).logits[:, -1].numpy()
    cos, sin = rotary_tables(TINY, 32)
    for tp in (1, 2):
        oracles = []
        for rank in range(tp):
            w = {k: v.double().numpy() for k, v in transform_weights(st, TINY, tp, rank).items()}
            w["rotary_cos"], w["rotary_sin"] = cos.double().numpy(), sin.double().numpy()
            oracles.append(GraphOracle(build_graph(TINY, capacity=32, tp_size=tp), w))
        if tp == 1:
            out = oracles[0].run({"input_ids": ids.numpy(), "positions": np.zeros(2, dtype=np.int64)})
            np.testing.assert_allclose(out["logits"], ref_prefill, rtol=1e-4, atol=1e-5)
            out = oracles[0].run({"input_ids": nxt.numpy(), "positions": np.full(2, 6, dtype=np.int64)})
            np.testing.assert_allclose(out["logits"], ref_decode, rtol=1e-4, atol=1e-5)
        else:
            # emulate the all_reduce: run both ranks node by node, summing partials
            _run_tp(oracles, ids.numpy(), np.zeros(2, dtype=np.int64), ref_prefill)
            _run_tp(oracles, nxt.numpy(), np.full(2, 6, dtype=np.int64), ref_decode)


def _run_tp(oracles, ids, pos, ref):
    envs = [dict(o.constants, input_ids=ids, positions=pos) for o in oracles]
    for idx, node in enumerate(oracles[0].graph["nodes"]):
        outs = []
        for o, env in zip(oracles, envs):
            n = o.graph["nodes"][idx]
            outs.append(o._op(n["op"], [env[x] for x in n["inputs"]], n.get("attrs", {})))
        if node["op"] == "tp_argmax":
            # vocab-parallel greedy pick over every rank's logits slice
            full = np.concatenate([np.asarray(env[node["inputs"][0]]) for env in envs], -1)
            outs = [[O.argmax(full)] for _ in envs]
        if node["op"] == "all_reduce_add_rms_norm":
            # sum the partials (input 1) over the ranks, then the residual add + norm
            total = sum(np.asarray(env[node["inputs"][1]]) for env in envs)
            outs = [o._op("add_rms_norm", [env[node["inputs"][0]], total, env[node["inputs"][2]]], node["attrs"])
                    for o, env in zip(oracles, envs)]
        if node["op"] == "linear_all_reduce_add_rms_norm":
            # each rank's partial projection of (input 1, input 2), summed over the ranks
            total = sum(O.linear(np.asarray(env[node["inputs"][1]]), np.asarray(env[node["inputs"][2]]), None)
                        for env in envs)
            outs = [o._op("add_rms_norm", [env[node["inputs"][0]], total, env[node["inputs"][3]]], node["attrs"])
                    for o, env in zip(oracles, envs)]
        for env, res in zip(envs, outs):
            for name, val in zip(node["outputs"], res):
                env[name] = val
    # vocab-parallel LM head: rank r holds logits columns [r*V/tp, (r+1)*V/tp)
    logits = np.concatenate([env["logits"] for env in envs], -1)
    np.testing.assert_allclose(logits, ref, rtol=1e-4, atol=1e-5)
    for env in envs:
        np.testing.assert_array_equal(env["next_ids"], np.argmax(ref, -1))


def test_vocab_parallel_lm_head_shards_recompose():
    """Under tensor parallelism the LM head is split by vocabulary rows (rank r holds
    ids [r*V/tp, (r+1)*V/tp)); tied embeddings keep the full table for the lookup.
    A vocabulary that does not divide evenly keeps a replicated head and argmax."""
    import dataclasses

    st = random_state(TINY, dtype=torch.float32, seed=4)
    full = transform_weights(st, TINY, 1, 0)
    shards = [transform_weights(st, TINY, 2, r) for r in range(2)]
    torch.testing.assert_close(torch.cat([s["lm_head"] for s in shards]), full["lm_head"])
    tied = dataclasses.replace(TINY, tie_embeddings=True)
    st_t = random_state(tied, dtype=torch.float32, seed=4)
    st_t.pop("lm_head.weight", None)
    sh = transform_weights(st_t, tied, 2, 1)
    assert sh["embed"].shape[0] == tied.vocab and sh["lm_head"].shape[0] == tied.vocab // 2
    torch.testing.assert_close(sh["lm_head"], st_t["model.embed_tokens.weight"][tied.vocab // 2:])
    odd = dataclasses.replace(TINY, vocab=51)
    assert [n["op"] for n in build_graph(odd, capacity=32, tp_size=2)["nodes"]][-1] == "argmax"
    assert transform_weights(random_state(odd, dtype=torch.float32), odd, 2, 0)["lm_head"].shape[0] == 51
