#!/usr/bin/env python3
"""Regenerate the committed golden fixtures under tests/golden/.

Run where the xdna-engine source tree is checked out (its path in XDNA_REF) and
`transformers` is importable:

    XDNA_REF=<path of the xdna-engine checkout> python tests/golden/make_golden.py

It writes
  bfp16_golden.npz  -- outputs of the reference's own numpy golden
                       route_b_kernels/ffn_bfp16/golden_ffn_gemm.py (to_bf16, to_bfp16_blocks,
                       gemm_bfp16), imported and run unchanged on seeded inputs;
  opt_hf_golden.npz -- greedy tokens + per-step logits of HuggingFace OPTForCausalLM (the
                       implementation the reference validates its opt-125m decode against,
                       scripts/opt125m_reference.py) on a small seeded random-init OPT whose
                       weights come from xdna_engine_b200.synth.make_opt_weights.
The known-answer values of the reference's Rust unit tests are transcribed by hand into
ref_kats.json (each entry cites its source file:line); this script does not touch that file.
The GPU box never runs this script: the tests only read the .npz files.
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
REF = os.environ.get("XDNA_REF", "")      # the xdna-engine checkout (needed only to regenerate)


def bfp16_fixture():
    path = os.path.join(REF, "route_b_kernels/ffn_bfp16/golden_ffn_gemm.py")
    spec = importlib.util.spec_from_file_location("golden_ffn_gemm", path)
    g = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(g)
    rng = np.random.default_rng(20240611)
    out = {}
    # activations ~N(0,1) and weights ~N(0, 1/sqrt(K)) as the golden's run_case draws them,
    # plus an N(0, 0.02) weight (the Whisper config's distribution) and edge rows.
    a = rng.standard_normal((8, 128)).astype(np.float32)
    b = (rng.standard_normal((128, 32)) / 11.3).astype(np.float32)
    w02 = (rng.standard_normal((64, 128)) * 0.02).astype(np.float32)
    edge = np.zeros((4, 64), np.float32)
    edge[1, :8] = [1.0, -1.0, 0.5, 0.25, 127.0, -128.0, 1e-3, 3.0]
    edge[2] = rng.standard_normal(64).astype(np.float32) * 1e-20
    edge[3, ::8] = 2.0 ** np.arange(-4, 4, dtype=np.float32)
    out["a"], out["b"], out["w02"], out["edge"] = a, b, w02, edge
    out["a_bf16"] = g.to_bf16(a)
    out["a_blocks_ax1"] = g.to_bfp16_blocks(g.to_bf16(a), axis=1)
    out["b_blocks_ax0"] = g.to_bfp16_blocks(g.to_bf16(b), axis=0)
    out["w02_blocks_ax0"] = g.to_bfp16_blocks(w02, axis=0)
    out["edge_blocks_ax1"] = g.to_bfp16_blocks(edge, axis=1)
    out["gemm_bfp16"] = g.gemm_bfp16(a, b)
    out["gemm_fp32"] = g.gemm_fp32(a, b)
    np.savez_compressed(os.path.join(HERE, "bfp16_golden.npz"), **out)
    print("bfp16_golden.npz:", {k: v.shape for k, v in out.items()})


OPT_SMALL = dict(n_layers=2, d_model=128, n_heads=2, head_dim=64, ffn=256, vocab=512,
                 max_pos=64, eps=1e-5)
OPT_SMALL_SEED = 7
OPT_SMALL_STD = 0.08


def opt_small_weights():
    from xdna_engine_b200.synth import OptConfig, make_opt_weights
    cfg = OptConfig(**OPT_SMALL)
    return cfg, make_opt_weights(cfg, seed=OPT_SMALL_SEED, std=OPT_SMALL_STD, bias_std=0.05,
                                 ln_std=0.1)


def weights_checksum(w):
    acc = np.float64(0.0)
    for k in ("emb_tok", "emb_pos", "lnf_w", "lnf_b"):
        acc += np.abs(w[k].astype(np.float64)).sum()
    for ly in w["layers"]:
        for v in ly.values():
            acc += np.abs(v.astype(np.float64)).sum()
    return acc


def opt_hf_fixture():
    import torch
    from transformers import OPTConfig, OPTForCausalLM
    cfg, w = opt_small_weights()
    hc = OPTConfig(vocab_size=cfg.vocab, hidden_size=cfg.d_model, num_hidden_layers=cfg.n_layers,
                   ffn_dim=cfg.ffn, num_attention_heads=cfg.n_heads,
                   max_position_embeddings=cfg.max_pos, do_layer_norm_before=True,
                   word_embed_proj_dim=cfg.d_model, activation_function="relu", dropout=0.0,
                   attention_dropout=0.0, enable_bias=True, layer_norm_elementwise_affine=True,
                   tie_word_embeddings=True, pad_token_id=1, bos_token_id=2, eos_token_id=2)
    model = OPTForCausalLM(hc).eval().float()
    sd = model.state_dict()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    new = {"model.decoder.embed_tokens.weight": t(w["emb_tok"]),
           "model.decoder.embed_positions.weight": t(w["emb_pos"]),
           "model.decoder.final_layer_norm.weight": t(w["lnf_w"]),
           "model.decoder.final_layer_norm.bias": t(w["lnf_b"]),
           "lm_head.weight": t(w["emb_tok"])}
    names = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
             "wo": "self_attn.out_proj", "w1": "fc1", "w2": "fc2"}
    bias = {"wq": "bq", "wk": "bk", "wv": "bv", "wo": "bo", "w1": "b1", "w2": "b2"}
    for i, ly in enumerate(w["layers"]):
        p = f"model.decoder.layers.{i}."
        for k, n in names.items():
            new[p + n + ".weight"] = t(ly[k].T)          # HF Linear is [out, in]
            new[p + n + ".bias"] = t(ly[bias[k]])
        new[p + "self_attn_layer_norm.weight"] = t(ly["ln1_w"])
        new[p + "self_attn_layer_norm.bias"] = t(ly["ln1_b"])
        new[p + "final_layer_norm.weight"] = t(ly["ln2_w"])
        new[p + "final_layer_norm.bias"] = t(ly["ln2_b"])
    missing = set(sd) - set(new)
    assert not missing, missing
    model.load_state_dict(new, strict=True)
    rng = np.random.default_rng(11)
    prompt = rng.integers(2, cfg.vocab, size=10, dtype=np.int64)
    n_new = 12
    ids = torch.from_numpy(prompt)[None]
    toks, logits = [], []
    with torch.no_grad():
        for _ in range(n_new):
            lg = model(input_ids=ids).logits[0, -1].float().numpy()
            nxt = int(np.argmax(lg))
            toks.append(nxt)
            logits.append(lg)
            ids = torch.cat([ids, torch.tensor([[nxt]])], dim=1)
    out = dict(prompt=prompt, tokens=np.array(toks, np.int64), logits=np.stack(logits),
               checksum=np.float64(weights_checksum(w)))
    np.savez_compressed(os.path.join(HERE, "opt_hf_golden.npz"), **out)
    print("opt_hf_golden.npz: tokens", toks)


BERT_SMALL = dict(n_layers=2, d_model=64, n_heads=2, ffn=128, vocab=300, max_pos=40, eps=1e-12,
                  pooling=0)
BERT_SMALL_SEED = 5


def bert_small_weights():
    from xdna_engine_b200.synth import BertConfig, make_bert_weights
    cfg = BertConfig(**BERT_SMALL)
    return cfg, make_bert_weights(cfg, seed=BERT_SMALL_SEED, std=0.1, bias_std=0.05, ln_std=0.1)


def bert_hf_fixture():
    """HF BertModel (what the reference validates BGE against, scripts/bge_reference.py):
    CLS row of last_hidden_state, L2-normalised, on a small seeded random BERT."""
    import torch
    from transformers import BertConfig as HFCfg, BertModel
    cfg, w = bert_small_weights()
    hc = HFCfg(vocab_size=cfg.vocab, hidden_size=cfg.d_model, num_hidden_layers=cfg.n_layers,
               num_attention_heads=cfg.n_heads, intermediate_size=cfg.ffn, hidden_act="gelu",
               hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0,
               max_position_embeddings=cfg.max_pos, type_vocab_size=2, layer_norm_eps=cfg.eps)
    model = BertModel(hc, add_pooling_layer=False).eval().float()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    sd = {"embeddings.word_embeddings.weight": t(w["word_emb"]),
          "embeddings.position_embeddings.weight": t(w["pos_emb"]),
          "embeddings.token_type_embeddings.weight": t(w["type_emb"]),
          "embeddings.LayerNorm.weight": t(w["emb_ln_w"]), "embeddings.LayerNorm.bias": t(w["emb_ln_b"])}
    m = {"q": "attention.self.query", "k": "attention.self.key", "v": "attention.self.value",
         "o": "attention.output.dense", "ffn1": "intermediate.dense", "ffn2": "output.dense"}
    for i, ly in enumerate(w["layers"]):
        p = f"encoder.layer.{i}."
        for k, n in m.items():
            sd[p + n + ".weight"] = t(ly[k + "_w"].T)
            sd[p + n + ".bias"] = t(ly[k + "_b"])
        sd[p + "attention.output.LayerNorm.weight"] = t(ly["attn_ln_w"])
        sd[p + "attention.output.LayerNorm.bias"] = t(ly["attn_ln_b"])
        sd[p + "output.LayerNorm.weight"] = t(ly["out_ln_w"])
        sd[p + "output.LayerNorm.bias"] = t(ly["out_ln_b"])
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("position_ids" in k or "token_type_ids" in k for k in missing), missing
    rng = np.random.default_rng(21)
    lens = np.array([1, 7, 19, 40], np.int32)
    ids = rng.integers(3, cfg.vocab, size=int(lens.sum())).astype(np.int32)
    embs, off = [], 0
    with torch.no_grad():
        for L in lens:
            x = torch.from_numpy(ids[off:off + L].astype(np.int64))[None]
            h = model(input_ids=x, token_type_ids=torch.zeros_like(x)).last_hidden_state[0, 0]
            embs.append(torch.nn.functional.normalize(h, dim=0).numpy())
            off += L
    np.savez_compressed(os.path.join(HERE, "bert_hf_golden.npz"), ids=ids, lens=lens, emb=np.stack(embs))
    print("bert_hf_golden.npz: ", np.stack(embs).shape)


WHISPER_SMALL = dict(n_layers=2, d_model=64, n_heads=2, ffn=128, n_mels=8, n_frames=20, max_src=10, eps=1e-5)
WHISPER_SMALL_SEED = 11


def whisper_small_weights():
    from xdna_engine_b200.synth import WhisperEncConfig, make_whisper_enc_weights, make_mel
    cfg = WhisperEncConfig(**WHISPER_SMALL)
    w = make_whisper_enc_weights(cfg, seed=WHISPER_SMALL_SEED, std=0.1, bias_std=0.05, ln_std=0.1)
    return cfg, w, make_mel(cfg, batch=2, seed=WHISPER_SMALL_SEED)


def whisper_hf_fixture():
    """HF WhisperEncoder (the model the reference's encoder.rs restates, weights from the same
    checkpoint layout): last_hidden_state on a small seeded random encoder, 2 clips."""
    import torch
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperEncoder
    cfg, w, mel = whisper_small_weights()
    hc = WhisperConfig(d_model=cfg.d_model, encoder_layers=cfg.n_layers, encoder_attention_heads=cfg.n_heads,
                       encoder_ffn_dim=cfg.ffn, num_mel_bins=cfg.n_mels, max_source_positions=cfg.max_src,
                       activation_function="gelu", dropout=0.0, attention_dropout=0.0, activation_dropout=0.0)
    model = WhisperEncoder(hc).eval().float()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    sd = {"conv1.weight": t(w["conv1_w"]), "conv1.bias": t(w["conv1_b"]),
          "conv2.weight": t(w["conv2_w"]), "conv2.bias": t(w["conv2_b"]),
          "embed_positions.weight": t(w["embed_positions"]),
          "layer_norm.weight": t(w["ln_post_w"]), "layer_norm.bias": t(w["ln_post_b"])}
    for i, ly in enumerate(w["layers"]):
        p = f"layers.{i}."
        for k, n in (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"),
                     ("out", "self_attn.out_proj"), ("fc1", "fc1"), ("fc2", "fc2")):
            sd[p + n + ".weight"] = t(ly[k + "_w"].T)
            if k != "k":
                sd[p + n + ".bias"] = t(ly[k + "_b"])
        sd[p + "self_attn_layer_norm.weight"] = t(ly["ln1_w"])
        sd[p + "self_attn_layer_norm.bias"] = t(ly["ln1_b"])
        sd[p + "final_layer_norm.weight"] = t(ly["ln2_w"])
        sd[p + "final_layer_norm.bias"] = t(ly["ln2_b"])
    missing, unexpected = model.load_state_dict(sd, strict=True), None
    with torch.no_grad():
        enc = model(torch.from_numpy(mel)).last_hidden_state.numpy()
    np.savez_compressed(os.path.join(HERE, "whisper_hf_golden.npz"), enc=enc)
    print("whisper_hf_golden.npz:", enc.shape)


WHISPER_DEC_SMALL = dict(n_layers=2, d_model=64, n_heads=2, ffn=128, vocab=300, max_tgt=40, n_enc=24)
WHISPER_DEC_SEED = 13
WHISPER_DEC_PROMPT = [1, 5, 7]


def whisper_dec_small():
    from xdna_engine_b200.synth import WhisperDecConfig, make_whisper_dec_weights, make_encoder_states
    cfg = WhisperDecConfig(**WHISPER_DEC_SMALL)
    w = make_whisper_dec_weights(cfg, seed=WHISPER_DEC_SEED, std=0.2, bias_std=0.05, ln_std=0.1)
    return cfg, w, make_encoder_states(cfg, 2, WHISPER_DEC_SEED)


def whisper_dec_hf_fixture():
    """HF WhisperDecoder + the tied proj_out (the model whisper_decoder.rs restates) on a small
    seeded decoder: greedy tokens and per-step logits for 2 streams after a 3-token prompt,
    recomputing the whole sequence each step (no cache)."""
    import torch
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperDecoder
    cfg, w, enc = whisper_dec_small()
    hc = WhisperConfig(d_model=cfg.d_model, decoder_layers=cfg.n_layers, decoder_attention_heads=cfg.n_heads,
                       decoder_ffn_dim=cfg.ffn, vocab_size=cfg.vocab, max_target_positions=cfg.max_tgt,
                       max_source_positions=cfg.n_enc, activation_function="gelu", dropout=0.0,
                       attention_dropout=0.0, activation_dropout=0.0, pad_token_id=0)
    model = WhisperDecoder(hc).eval().float()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    sd = {"embed_tokens.weight": t(w["embed_tokens"]), "embed_positions.weight": t(w["embed_positions"]),
          "layer_norm.weight": t(w["ln_post_w"]), "layer_norm.bias": t(w["ln_post_b"])}
    names = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "out": "self_attn.out_proj",
             "cross_q": "encoder_attn.q_proj", "cross_k": "encoder_attn.k_proj", "cross_v": "encoder_attn.v_proj",
             "cross_out": "encoder_attn.out_proj", "fc1": "fc1", "fc2": "fc2"}
    for i, ly in enumerate(w["layers"]):
        p = f"layers.{i}."
        for k, n in names.items():
            sd[p + n + ".weight"] = t(ly[k + "_w"].T)
            if k not in ("k", "cross_k"):
                sd[p + n + ".bias"] = t(ly[k + "_b"])
        for a, b in (("ln_self", "self_attn_layer_norm"), ("ln_cross", "encoder_attn_layer_norm"),
                     ("ln_final", "final_layer_norm")):
            sd[p + b + ".weight"] = t(ly[a + "_w"])
            sd[p + b + ".bias"] = t(ly[a + "_b"])
    model.load_state_dict(sd, strict=True)
    n_new = 12
    toks = np.zeros((2, n_new), np.int64)
    lgs = np.zeros((2, n_new, cfg.vocab), np.float32)
    with torch.no_grad():
        for b in range(2):
            seq = list(WHISPER_DEC_PROMPT)
            for s in range(n_new):
                h = model(input_ids=torch.tensor([seq]), encoder_hidden_states=t(enc[b:b + 1])).last_hidden_state
                lg = (h[0, -1] @ t(w["embed_tokens"]).T).numpy()
                lgs[b, s] = lg
                toks[b, s] = int(np.argmax(lg))
                seq.append(int(toks[b, s]))
    np.savez_compressed(os.path.join(HERE, "whisper_dec_hf_golden.npz"), tokens=toks, logits=lgs)
    print("whisper_dec_hf_golden.npz:", toks.tolist())


GEMMA_SMALL = dict(n_layers=7, d_model=256, n_q_heads=4, head_dim=64, ffn=512, vocab=500, window=8)
GEMMA_SEED = 1
GEMMA_PROMPT = [2, 3, 4, 5, 6, 7, 8, 9, 10, 11]


def gemma_small():
    from xdna_engine_b200.synth import GemmaConfig, make_gemma_weights
    cfg = GemmaConfig(**GEMMA_SMALL)
    return cfg, make_gemma_weights(cfg, seed=GEMMA_SEED, std=0.2, norm_std=0.1, embed_std=0.01)


def gemma_hf_fixture():
    """HF Gemma3ForCausalLM (the model rust/npu-gemma ports) on a small seeded config with a
    sliding window of 8 and the 5:1 local:global pattern: greedy tokens and logits."""
    import torch
    from transformers import Gemma3TextConfig, Gemma3ForCausalLM
    cfg, w = gemma_small()
    types = ["full_attention" if (i + 1) % cfg.pattern == 0 else "sliding_attention" for i in range(cfg.n_layers)]
    hc = Gemma3TextConfig(vocab_size=cfg.vocab, hidden_size=cfg.d_model, intermediate_size=cfg.ffn,
                          num_hidden_layers=cfg.n_layers, num_attention_heads=cfg.n_q_heads, num_key_value_heads=1,
                          head_dim=cfg.head_dim, sliding_window=cfg.window, layer_types=types,
                          query_pre_attn_scalar=int(cfg.query_pre_attn_scalar), rms_norm_eps=cfg.eps,
                          rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": cfg.theta_local},
                                           "full_attention": {"rope_type": "default", "rope_theta": cfg.theta_global}},
                          max_position_embeddings=64, attn_implementation="eager", tie_word_embeddings=True)
    model = Gemma3ForCausalLM(hc).eval().float()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    sd = {"model.embed_tokens.weight": t(w["embed"]), "model.norm.weight": t(w["final_norm"]),
          "lm_head.weight": t(w["embed"])}
    names = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj",
             "wg": "mlp.gate_proj", "wu": "mlp.up_proj", "wd": "mlp.down_proj"}
    norms = {"in_norm": "input_layernorm", "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm",
             "post_attn_norm": "post_attention_layernorm", "pre_ffn_norm": "pre_feedforward_layernorm",
             "post_ffn_norm": "post_feedforward_layernorm"}
    for i, ly in enumerate(w["layers"]):
        p = f"model.layers.{i}."
        for k, n in names.items():
            sd[p + n + ".weight"] = t(ly[k].T)
        for k, n in norms.items():
            sd[p + n + ".weight"] = t(ly[k])
    model.load_state_dict(sd, strict=True)
    seq = list(GEMMA_PROMPT)
    n_new = 12
    toks, lgs = [], []
    with torch.no_grad():
        for _ in range(n_new):
            lg = model(input_ids=torch.tensor([seq])).logits[0, -1].numpy()
            lgs.append(lg)
            toks.append(int(np.argmax(lg)))
            seq.append(toks[-1])
    np.savez_compressed(os.path.join(HERE, "gemma_hf_golden.npz"), tokens=np.array(toks), logits=np.stack(lgs))
    print("gemma_hf_golden.npz:", toks)


def _load_ref_module(rel, name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


PK_DW_CHANNELS = np.array([0, 1, 2, 3, 100, 255, 256, 511, 512, 700, 777, 900, 1000, 1021, 1022, 1023])


def parakeet_fixture():
    """Outputs of the reference's own Parakeet numpy goldens on seeded synthetic inputs:
    rel_shift_host / rel_shift_strided (scripts/parakeet_relpos_mha_golden.py:59-75), the fp32
    depthwise conv 'same' host_reference (route_b_kernels/dwconv1d/golden_dwconv1d_k9.py:40-48;
    its module fixes C = 1024, T = 400, k = 9: 16 channels are stored, plus the f64 sum of all)
    and conv2d_ref (route_b_kernels/subsample_conv2d/golden_subsample.py:58-79, f64)."""
    rs = _load_ref_module("scripts/parakeet_relpos_mha_golden.py", "pk_relpos")
    dwm = _load_ref_module("route_b_kernels/dwconv1d/golden_dwconv1d_k9.py", "pk_dw")
    ssm = _load_ref_module("route_b_kernels/subsample_conv2d/golden_subsample.py", "pk_sub")
    rng = np.random.default_rng(77)
    out = {}
    for T in (1, 2, 9, 31):
        bd = rng.standard_normal((3, T, 2 * T - 1)).astype(np.float32)
        out[f"bd_{T}"] = bd
        out[f"shift_{T}"] = rs.rel_shift_host(bd)
        assert np.array_equal(out[f"shift_{T}"], rs.rel_shift_strided(bd))
    x = np.random.default_rng(78).standard_normal((dwm.C, dwm.T)).astype(np.float32)
    dw = (np.random.default_rng(79).standard_normal((dwm.C, dwm.K)) / 3).astype(np.float32)
    db = (np.random.default_rng(80).standard_normal(dwm.C) * 0.02).astype(np.float32)
    y = dwm.host_reference(x, dw, db)
    out["dw_out"] = y[PK_DW_CHANNELS]
    out["dw_sum"] = np.array(np.sum(y.astype(np.float64)))
    cases = [((2, 9, 10), (4, 2, 3, 3), 2, 1, 1), ((4, 9, 10), (4, 1, 3, 3), 2, 1, 4),
             ((4, 5, 6), (3, 4, 1, 1), 1, 0, 1), ((1, 12, 8), (5, 1, 3, 3), 2, 1, 1)]
    for i, (xs, ws, st, pd, g) in enumerate(cases):
        xi = rng.standard_normal(xs).astype(np.float32)
        wi = (rng.standard_normal(ws) * 0.3).astype(np.float32)
        bi = (rng.standard_normal(ws[0]) * 0.1).astype(np.float32)
        out[f"c2d_x{i}"], out[f"c2d_w{i}"], out[f"c2d_b{i}"] = xi, wi, bi
        out[f"c2d_y{i}"] = ssm.conv2d_ref(xi.astype(np.float64), wi.astype(np.float64), bi.astype(np.float64),
                                          st, pd, g)
        out[f"c2d_meta{i}"] = np.array([st, pd, g])
    np.savez_compressed(os.path.join(HERE, "parakeet_golden.npz"), **out)
    print("parakeet_golden.npz:", len(out), "arrays")


if __name__ == "__main__":
    if not REF or not os.path.isdir(REF):
        sys.exit("make_golden.py: set XDNA_REF to the xdna-engine source checkout")
    import sys
    only = set(sys.argv[1:])
    if not only or "gemma" in only:
        gemma_hf_fixture()
    if not only or "whisper_dec" in only:
        whisper_dec_hf_fixture()
    if not only or "parakeet" in only:
        parakeet_fixture()
    if not only or "bfp16" in only:
        bfp16_fixture()
    if not only or "opt" in only:
        opt_hf_fixture()
    if not only or "bert" in only:
        bert_hf_fixture()
    if not only or "whisper" in only:
        whisper_hf_fixture()
