"""The TP Llama decoder on the native kernels vs a plain PyTorch fp32 forward
of the same random weights (logit cosine / top-1 agreement), chunked prefill
consistency, and CUDA-graph decode vs eager decode."""

import pytest
import torch
import torch.nn.functional as F

from conftest import sub

pytestmark = pytest.mark.gpu


def torch_forward(w, cfg, ids):
    """fp32 reference forward of the full sequence (no cache); returns the
    final normalised hidden states [T, H]."""
    ref = sub("ops.reference")
    T = len(ids)
    D, nq, nkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    cs = sub("ops").rope_cos_sin(cfg.max_pos, D, cfg.rope_theta, "cuda")
    pos = torch.arange(T, device="cuda", dtype=torch.int32)
    h = w.embed.float()[torch.tensor(ids, device="cuda")]
    x = ref.rmsnorm(h, w.layers[0]["ln1"], cfg.eps)
    res = h
    for li, L in enumerate(w.layers):
        qkv = x @ L["qkv"].float().t()
        q = qkv[:, : nq * D].view(T, nq, D)
        k = qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D)
        v = qkv[:, (nq + nkv) * D:].view(T, nkv, D)
        q, k = ref.rope(q, pos, cs), ref.rope(k, pos, cs)
        o = ref.attention(q, k, v, causal_offset=0).reshape(T, nq * D)
        res = res + o @ L["o"].float().t()
        x = ref.rmsnorm(res, L["ln2"], cfg.eps)
        gu = x @ L["gate_up"].float().t()
        g, u = gu.chunk(2, -1)
        res = res + (F.silu(g) * u) @ L["down"].float().t()
        nxt = w.layers[li + 1]["ln1"] if li + 1 < len(w.layers) else w.norm
        x = ref.rmsnorm(res, nxt, cfg.eps)
    return x


def test_prefill_matches_torch_reference():
    models, eng_mod = sub("models"), sub("engine")
    cfg = models.LlamaConfig.tiny()
    eng = eng_mod.LLMEngine(cfg, max_batch=4, max_seq=512, chunk=64, seed=3, use_graphs=False)
    prompt = torch.randint(0, cfg.vocab, (150,), generator=torch.Generator().manual_seed(0)).tolist()
    req = eng.add_request(prompt, 1)
    eng.sched._admit()
    eng._sync_block_row(req)
    slots = eng.kv.slots(req.blocks, 0, len(prompt))
    # native, chunked in pieces of 64 (+22), hidden state of the last token
    hid = None
    for s in range(0, len(prompt), 64):
        n = min(64, len(prompt) - s)
        dev = eng.device
        ids = torch.tensor(prompt[s:s + n], dtype=torch.int32, device=dev)
        pos = torch.arange(s, s + n, dtype=torch.int32, device=dev)
        sl = torch.tensor(slots[s:s + n], dtype=torch.int64, device=dev)
        cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
        kvl = torch.tensor([s + n], dtype=torch.int32, device=dev)
        bt = eng.block_table[req.slot:req.slot + 1]
        tiles = sub("ops").prefill_tiles([n]).to(dev)
        last = torch.tensor([n - 1], dtype=torch.int64, device=dev)
        attn = lambda li, q, kc, vc: sub("ops").prefill_attention(q, kc, vc, cu, kvl, bt, tiles, eng.model.scale)
        hid = eng.model.forward(ids, pos, sl, eng.kv.caches, attn, last, return_hidden=True)
    want = torch_forward(eng.weights, cfg, prompt)[-1]
    got = hid[0].float()
    cos = F.cosine_similarity(got, want, dim=0).item()
    assert cos > 0.995, cos
    logits_got = got @ eng.weights.lm_head.float().t()
    logits_want = want @ eng.weights.lm_head.float().t()
    top = logits_want.topk(5).indices
    assert logits_got.argmax().item() in top.tolist()


def test_generate_graphs_match_eager():
    models, eng_mod = sub("models"), sub("engine")
    cfg = models.LlamaConfig.tiny()
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (17, 64, 130)]
    outs = []
    for graphs in (False, True):
        eng = eng_mod.LLMEngine(cfg, max_batch=8, max_seq=512, chunk=64, seed=5, use_graphs=graphs,
                                graph_sizes=(1, 8))
        outs.append(eng.generate(prompts, max_new_tokens=12))
    assert outs[0] == outs[1]
    assert all(len(o) == 12 for o in outs[0])


def test_chunk_size_does_not_change_hidden_state():
    """Prefilling a prompt in 32-token or 1024-token chunks gives the same last
    hidden state up to bf16 noise (the kernels see the same keys per query,
    grouped differently)."""
    models, eng_mod = sub("models"), sub("engine")
    ops = sub("ops")
    cfg = models.LlamaConfig.tiny()
    prompt = list(range(1, 200))
    hid = []
    for chunk in (32, 1024):
        eng = eng_mod.LLMEngine(cfg, max_batch=4, max_seq=512, chunk=chunk, seed=9, use_graphs=False)
        req = eng.add_request(prompt, 1)
        eng.sched._admit()
        eng._sync_block_row(req)
        slots = eng.kv.slots(req.blocks, 0, len(prompt))
        dev = eng.device
        h = None
        for s0 in range(0, len(prompt), chunk):
            n = min(chunk, len(prompt) - s0)
            ids = torch.tensor(prompt[s0:s0 + n], dtype=torch.int32, device=dev)
            pos = torch.arange(s0, s0 + n, dtype=torch.int32, device=dev)
            sl = torch.tensor(slots[s0:s0 + n], dtype=torch.int64, device=dev)
            cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
            kvl = torch.tensor([s0 + n], dtype=torch.int32, device=dev)
            bt = eng.block_table[req.slot:req.slot + 1]
            tiles = ops.prefill_tiles([n]).to(dev)
            last = torch.tensor([n - 1], dtype=torch.int64, device=dev)
            attn = lambda li, q, kc, vc: ops.prefill_attention(q, kc, vc, cu, kvl, bt, tiles, eng.model.scale)
            h = eng.model.forward(ids, pos, sl, eng.kv.caches, attn, last, return_hidden=True)
        hid.append(h[0].float())
    cos = F.cosine_similarity(hid[0], hid[1], dim=0).item()
    assert cos > 0.999, cos


def test_prefill_graph_matches_eager():
    """Full single-request chunks replayed from a captured graph give the same
    tokens as the eager chunk forwards (partial last chunks stay eager)."""
    models, eng_mod = sub("models"), sub("engine")
    cfg = models.LlamaConfig.tiny()
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (128, 200, 64)]
    res = []
    for pg in (False, True):
        eng = eng_mod.LLMEngine(cfg, max_batch=4, max_seq=512, chunk=64, seed=13, use_graphs=False,
                                prefill_graph=pg)
        res.append(eng.generate(prompts, max_new_tokens=5))
        if pg:
            assert eng.prefill_graph.graph is not None
    assert res[0] == res[1]


def test_http_server_matches_generate():
    """The OpenAI-style front end drives the real engine: token-id prompts
    posted one after another come back with the same greedy tokens as
    ``generate`` of each prompt alone on the same weights (same batches, so
    the same kernels run)."""
    requests = pytest.importorskip("requests")
    import threading

    from conftest import free_port

    models, eng_mod, srv_mod = sub("models"), sub("engine"), sub("server")
    cfg = models.LlamaConfig.tiny()
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=torch.Generator().manual_seed(n)).tolist()
               for n in (40, 130, 7)]
    ref = eng_mod.LLMEngine(cfg, max_batch=4, max_seq=512, chunk=64, seed=21, use_graphs=False)
    want = [ref.generate([p], max_new_tokens=6)[0] for p in prompts]
    eng = eng_mod.LLMEngine(cfg, max_batch=4, max_seq=512, chunk=64, seed=21, use_graphs=False)
    server = srv_mod.EngineServer(eng, max_prompt=512)
    port = free_port()
    http, _ = srv_mod.start_http(srv_mod.build_app(server, cfg.name), "127.0.0.1", port)
    got = [None] * len(prompts)

    def clients():
        try:
            for i in range(len(prompts)):
                r = requests.post(f"http://127.0.0.1:{port}/v1/completions",
                                  json={"prompt": prompts[i], "max_tokens": 6}, timeout=120)
                got[i] = r.json()["choices"][0]["token_ids"]
        finally:
            server.stop()

    threading.Thread(target=clients, daemon=True).start()
    try:
        server.serve_forever()  # CUDA work stays on this thread
    finally:
        http.should_exit = True
    assert got == want


def _engine_last_hidden(eng, prompt, chunk):
    """Last token's final hidden state, prefilled chunk by chunk."""
    ops = sub("ops")
    req = eng.add_request(prompt, 1)
    eng.sched._admit()
    eng._sync_block_row(req)
    slots = eng.kv.slots(req.blocks, 0, len(prompt))
    dev = eng.device
    hid = None
    for s in range(0, len(prompt), chunk):
        n = min(chunk, len(prompt) - s)
        ids = torch.tensor(prompt[s:s + n], dtype=torch.int32, device=dev)
        pos = torch.arange(s, s + n, dtype=torch.int32, device=dev)
        sl = torch.tensor(slots[s:s + n], dtype=torch.int64, device=dev)
        cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
        kvl = torch.tensor([s + n], dtype=torch.int32, device=dev)
        bt = eng.block_table[req.slot:req.slot + 1]
        tiles = ops.prefill_tiles([n]).to(dev)
        last = torch.tensor([n - 1], dtype=torch.int64, device=dev)
        attn = lambda li, q, kc, vc: ops.prefill_attention(q, kc, vc, cu, kvl, bt, tiles, eng.model.scale)  # noqa
        hid = eng.model.forward(ids, pos, sl, eng.kv.caches, attn, last, return_hidden=True)
    return hid[0].float()


def test_hf_checkpoint_engine_matches_reference(tmp_path):
    """A Hugging Face-layout safetensors checkpoint (separate q/k/v and
    gate/up projections, Llama 3.1 RoPE scaling, tied embeddings) loaded with
    LLMEngine.from_pretrained gives the same last hidden state as an fp32
    forward written directly over the checkpoint's tensors."""
    import json

    models, eng_mod, ops, ref = sub("models"), sub("engine"), sub("ops"), sub("ops.reference")
    H, D, nq, nkv, Fd, V, NL = 512, 128, 8, 2, 1024, 4096, 2
    scaling = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
               "original_max_position_embeddings": 64}
    cfg_json = {"hidden_size": H, "num_hidden_layers": NL, "num_attention_heads": nq, "num_key_value_heads": nkv,
                "head_dim": D, "intermediate_size": Fd, "vocab_size": V, "rope_theta": 500000.0,
                "rms_norm_eps": 1e-5, "max_position_embeddings": 1024, "rope_scaling": scaling,
                "tie_word_embeddings": True}
    g = torch.Generator().manual_seed(1)
    rnd = lambda *s: (torch.randn(*s, generator=g) * 0.05).to(torch.bfloat16)  # noqa: E731
    one = lambda n: (1 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16)  # noqa: E731
    t = {"model.embed_tokens.weight": rnd(V, H) * 20, "model.norm.weight": one(H)}
    for i in range(NL):
        p = f"model.layers.{i}."
        t.update({p + "input_layernorm.weight": one(H), p + "post_attention_layernorm.weight": one(H),
                  p + "self_attn.q_proj.weight": rnd(nq * D, H), p + "self_attn.k_proj.weight": rnd(nkv * D, H),
                  p + "self_attn.v_proj.weight": rnd(nkv * D, H), p + "self_attn.o_proj.weight": rnd(H, nq * D),
                  p + "mlp.gate_proj.weight": rnd(Fd, H), p + "mlp.up_proj.weight": rnd(Fd, H),
                  p + "mlp.down_proj.weight": rnd(H, Fd)})
    models.write_safetensors(str(tmp_path / "model.safetensors"), t)
    (tmp_path / "config.json").write_text(json.dumps(cfg_json))
    eng = eng_mod.LLMEngine.from_pretrained(str(tmp_path), max_batch=2, max_seq=512, chunk=64, use_graphs=False)
    prompt = torch.randint(0, V, (150,), generator=torch.Generator().manual_seed(2)).tolist()
    got = _engine_last_hidden(eng, prompt, 64)

    c = {k: v.cuda().float() for k, v in t.items()}
    T = len(prompt)
    cs = ops.rope_cos_sin(1024, D, 500000.0, "cuda", scaling)
    pos = torch.arange(T, device="cuda", dtype=torch.int32)
    res = c["model.embed_tokens.weight"][torch.tensor(prompt, device="cuda")]
    for i in range(NL):
        p = f"model.layers.{i}."
        x = ref.rmsnorm(res, c[p + "input_layernorm.weight"], 1e-5)
        q = (x @ c[p + "self_attn.q_proj.weight"].t()).view(T, nq, D)
        k = (x @ c[p + "self_attn.k_proj.weight"].t()).view(T, nkv, D)
        v = (x @ c[p + "self_attn.v_proj.weight"].t()).view(T, nkv, D)
        q, k = ref.rope(q, pos, cs), ref.rope(k, pos, cs)
        o = ref.attention(q, k, v, causal_offset=0).reshape(T, nq * D)
        res = res + o @ c[p + "self_attn.o_proj.weight"].t()
        x = ref.rmsnorm(res, c[p + "post_attention_layernorm.weight"], 1e-5)
        a = F.silu(x @ c[p + "mlp.gate_proj.weight"].t()) * (x @ c[p + "mlp.up_proj.weight"].t())
        res = res + a @ c[p + "mlp.down_proj.weight"].t()
    want = ref.rmsnorm(res, c["model.norm.weight"], 1e-5)[-1]
    assert F.cosine_similarity(got, want, dim=0).item() > 0.995
    logits_want = want @ c["model.embed_tokens.weight"].t()  # tied LM head
    assert (got @ c["model.embed_tokens.weight"].t()).argmax().item() in logits_want.topk(5).indices.tolist()


@pytest.mark.gpu
def test_awq_checkpoint_dequantizes_on_device(tmp_path):
    """An AWQ int4 checkpoint (the reference's served model format) loads with
    each shard dequantized on the GPU: the bf16 shards equal the CPU
    dequantization bit for bit, and the engine serves from them."""
    import json

    models, eng_mod = sub("models"), sub("engine")
    H, D, nq, nkv, Fd, V, NL, G = 512, 128, 8, 2, 1024, 4096, 2, 128
    cfg_json = {"architectures": ["LlamaForCausalLM"], "hidden_size": H, "num_hidden_layers": NL,
                "num_attention_heads": nq, "num_key_value_heads": nkv, "head_dim": D, "intermediate_size": Fd,
                "vocab_size": V, "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "max_position_embeddings": 1024,
                "quantization_config": {"quant_method": "awq", "bits": 4, "group_size": G, "zero_point": True,
                                        "version": "gemm"}}
    g = torch.Generator().manual_seed(3)
    rnd = lambda *s: (torch.randn(*s, generator=g) * 0.05).to(torch.float16)  # noqa: E731
    t = {"model.embed_tokens.weight": rnd(V, H) * 20, "model.norm.weight": torch.ones(H, dtype=torch.float16),
         "lm_head.weight": rnd(V, H)}
    shapes = {"self_attn.q_proj": (nq * D, H), "self_attn.k_proj": (nkv * D, H), "self_attn.v_proj": (nkv * D, H),
              "self_attn.o_proj": (H, nq * D), "mlp.gate_proj": (Fd, H), "mlp.up_proj": (Fd, H),
              "mlp.down_proj": (H, Fd)}
    for i in range(NL):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = torch.ones(H, dtype=torch.float16)
        t[p + "post_attention_layernorm.weight"] = torch.ones(H, dtype=torch.float16)
        for name, shape in shapes.items():
            qw, qz, s = models.awq_quantize(rnd(*shape), G)
            t[p + name + ".qweight"], t[p + name + ".qzeros"], t[p + name + ".scales"] = qw, qz, s
    models.write_safetensors(str(tmp_path / "model.safetensors"), t)
    (tmp_path / "config.json").write_text(json.dumps(cfg_json))
    _, w_gpu = models.load_llama(str(tmp_path), 0, 1, "cuda")
    _, w_cpu = models.load_llama(str(tmp_path), 0, 1, "cpu")
    for L_g, L_c in zip(w_gpu.layers, w_cpu.layers):
        for k in ("qkv", "o", "gate_up", "down"):
            assert L_g[k].is_cuda and torch.equal(L_g[k].cpu(), L_c[k]), k
    eng = eng_mod.LLMEngine.from_pretrained(str(tmp_path), max_batch=2, max_seq=512, chunk=64, use_graphs=False)
    out = eng.generate([list(range(1, 40))], max_new_tokens=4)[0]
    assert len(out) == 4 and all(0 <= x < V for x in out)
