"""HF safetensors checkpoint with fp8 e4m3 weights + fp32 128x128 block
scales (`weight_scale_inv`), loaded into MXFP8 serving weights (CPU path)."""
import torch


def test_fp8_checkpoint_roundtrip(tmp_path):
    from b200ds import EngineConfig, SamplingParams, load_engine
    from b200ds.config import ModelConfig, tiny_config
    from b200ds.models.loader import load_checkpoint, save_checkpoint_fp8
    from b200ds.models.reference import ReferenceModel, init_weights
    cfg = tiny_config(dense_format="mxfp8", expert_format="mxfp8")
    sd = init_weights(cfg, 0)
    save_checkpoint_fp8(sd, str(tmp_path), cfg)
    # config.json round trip
    cfg2 = ModelConfig.from_hf(str(tmp_path / "config.json"))
    assert cfg2.hidden_size == cfg.hidden_size and cfg2.n_routed_experts == cfg.n_routed_experts
    ck = load_checkpoint(str(tmp_path))
    assert ck["model.layers.0.self_attn.o_proj.weight"].dtype == torch.float8_e4m3fn
    assert "model.layers.0.self_attn.o_proj.weight_scale_inv" in ck
    # oracle on the checkpoint's dequantized weights
    deq = {}
    for k, v in ck.items():
        if k.endswith("_scale_inv"):
            continue
        s = ck.get(k + "_scale_inv")
        if s is not None:
            N, K = v.shape
            v = v.float() * s.repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
        deq[k] = v.float()
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab_size, (2, 16), generator=g)
    oracle = ReferenceModel(cfg, deq)
    otoks, ologits = oracle.greedy(prompts, 4)
    eng = load_engine(cfg, weights=str(tmp_path), ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    # served MXFP8 weights = the checkpoint's weights up to one MXFP8 requantization
    lw = eng.model.layers[0]
    o_srv = lw.attn.o_proj.w.dequant()[: cfg.hidden_size]
    o_ck = deq["model.layers.0.self_attn.o_proj.weight"]
    assert ((o_srv - o_ck).norm() / o_ck.norm()).item() < 0.03
    w13 = eng.model.layers[1].ffn.experts.w13
    from b200ds.ops.quant import dequant_mxfp8
    e0 = dequant_mxfp8(w13.data[0], w13.sf[0])
    ck0 = torch.cat([deq["model.layers.1.mlp.experts.0.gate_proj.weight"], deq["model.layers.1.mlp.experts.0.up_proj.weight"]])
    assert ((e0 - ck0).norm() / ck0.norm()).item() < 0.03
    logs = []
    orig = eng.model.forward
    eng.model.forward = lambda fb: logs.append(orig(fb)) or logs[-1]
    eng.generate(prompts.tolist(), SamplingParams(max_tokens=4))
    # MXFP8 weights *and* activations through 2 layers of a hidden-256 model:
    # close to the fp32 oracle, not equal
    rel = ((logs[0] - ologits[0]).norm() / ologits[0].norm()).item()
    assert rel < 0.25, rel


def test_mtp_layer_from_checkpoint(tmp_path):
    """A checkpoint with DeepSeek-V3's MTP layer (layer num_hidden_layers:
    enorm / hnorm / eh_proj / decoder layer / shared_head.norm, fp8 blocks)
    loads as the speculative draft; MTP decoding gives the greedy tokens."""
    from b200ds import EngineConfig, SamplingParams, load_engine
    from b200ds.config import ModelConfig, tiny_config
    from b200ds.models.loader import save_checkpoint_fp8
    from b200ds.models.reference import init_weights
    cfg = tiny_config(dense_format="mxfp8", expert_format="mxfp8", num_nextn_predict_layers=1)
    save_checkpoint_fp8(init_weights(cfg, 0), str(tmp_path), cfg)
    assert ModelConfig.from_hf(str(tmp_path / "config.json")).num_nextn_predict_layers == 1
    prompts = torch.randint(0, cfg.vocab_size, (2, 12), generator=torch.Generator().manual_seed(2)).tolist()
    outs = {}
    for mtp in (False, True):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, spec_mtp=mtp, spec_k=2)
        eng = load_engine(cfg, weights=str(tmp_path), ecfg=ecfg, device="cpu")
        assert eng.model.mtp is not None
        outs[mtp] = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=6))]
    assert outs[True] == outs[False]


def test_lazy_checkpoint_reads_only_this_ranks_weights(tmp_path):
    """The checkpoint is read on access: an EP rank building its model reads
    its own experts' tensors and none of the other ranks' experts."""
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.models.loader import LazyCheckpoint, build_model, save_checkpoint_fp8
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState
    cfg = tiny_config()
    save_checkpoint_fp8(init_weights(cfg, 0), str(tmp_path), cfg)
    ck = LazyCheckpoint(str(tmp_path))
    assert ck.reads == 0 and len(ck) > 0
    seen = []
    orig = LazyCheckpoint.__getitem__

    def spy(self, k):
        seen.append(k)
        return orig(self, k)
    LazyCheckpoint.__getitem__ = spy
    try:
        ps = ParallelState(world_size=2, rank=1, tp_size=2, ep_size=2, tp_rank=1, ep_rank=1)
        build_model(cfg, EngineConfig(page_size=8, cuda_graphs=False, tp_size=2, ep_size=2), ps, ck, device="cpu")
    finally:
        LazyCheckpoint.__getitem__ = orig
    experts = {int(k.split(".experts.")[1].split(".")[0]) for k in seen if ".experts." in k}
    per = cfg.n_routed_experts // 2
    assert experts == set(range(per, 2 * per))


def test_deepseek_v3_hf_config_json():
    """The published DeepSeek-V3 config.json fields map onto the 671B preset
    (fp8 checkpoint -> MXFP8 serving formats; unknown keys ignored)."""
    from b200ds.config import ModelConfig, PRESETS
    d = {"architectures": ["DeepseekV3ForCausalLM"], "model_type": "deepseek_v3", "vocab_size": 129280,
         "hidden_size": 7168, "intermediate_size": 18432, "moe_intermediate_size": 2048, "num_hidden_layers": 61,
         "num_nextn_predict_layers": 1, "num_attention_heads": 128, "num_key_value_heads": 128,
         "n_shared_experts": 1, "n_routed_experts": 256, "ep_size": 1, "routed_scaling_factor": 2.5,
         "kv_lora_rank": 512, "q_lora_rank": 1536, "qk_rope_head_dim": 64, "v_head_dim": 128,
         "qk_nope_head_dim": 128, "topk_method": "noaux_tc", "n_group": 8, "topk_group": 4,
         "num_experts_per_tok": 8, "moe_layer_freq": 1, "first_k_dense_replace": 3, "norm_topk_prob": True,
         "scoring_func": "sigmoid", "hidden_act": "silu", "max_position_embeddings": 163840, "rms_norm_eps": 1e-6,
         "rope_theta": 10000, "rope_scaling": {"beta_fast": 32, "beta_slow": 1, "factor": 40, "mscale": 1.0,
                                               "mscale_all_dim": 1.0, "original_max_position_embeddings": 4096,
                                               "type": "yarn"},
         "tie_word_embeddings": False, "torch_dtype": "bfloat16", "bos_token_id": 0, "eos_token_id": 1,
         "quantization_config": {"activation_scheme": "dynamic", "fmt": "e4m3", "quant_method": "fp8",
                                 "weight_block_size": [128, 128]}}
    c = ModelConfig.from_hf(d)
    p = PRESETS["deepseek-v3-671b"]()
    for f in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads", "q_lora_rank", "kv_lora_rank",
              "qk_nope_head_dim", "qk_rope_head_dim", "v_head_dim", "n_routed_experts", "num_experts_per_tok",
              "n_group", "topk_group", "first_k_dense_replace", "moe_intermediate_size", "intermediate_size"):
        assert getattr(c, f) == getattr(p, f), f
    assert c.dense_format == c.expert_format == "mxfp8" and c.num_nextn_predict_layers == 1
    assert abs(c.softmax_scale - p.softmax_scale) < 1e-9 and c.rope_scaling["factor"] == 40
    assert 600e9 < c.num_params() < 700e9


def test_checkpoint_dir_sets_eos(tmp_path):
    import json
    from b200ds import EngineConfig, load_engine
    from b200ds.config import tiny_config
    from b200ds.models.loader import save_checkpoint_fp8
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    save_checkpoint_fp8(init_weights(cfg, 0), str(tmp_path), cfg)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [7, 9]}))
    eng = load_engine(str(tmp_path), ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    assert eng.eos == 7


def test_dequant_blocked_block_shapes():
    """Block scales of 128 x 128 (fp32) and 32 x 32 (UE8M0 bytes) with ragged
    edges: each element is multiplied by its own block's scale."""
    from b200ds.ops.quant import block_scales_float, dequant_blocked
    g = torch.Generator().manual_seed(3)
    for (N, K, b) in ((300, 200, 128), (70, 96, 32), (64, 33, 32)):
        w = (torch.randn(N, K, generator=g) * 50).to(torch.float8_e4m3fn)
        nb, kb = (N + b - 1) // b, (K + b - 1) // b
        if b == 32:
            e = torch.randint(120, 134, (nb, kb), generator=g).to(torch.uint8)
            s = e.view(torch.float8_e8m0fnu)
            sf = torch.pow(2.0, e.float() - 127)
            assert torch.equal(block_scales_float(s), sf) and torch.equal(block_scales_float(e), sf)
        else:
            s = torch.rand(nb, kb, generator=g) + 0.5
            sf = s
        want = torch.empty(N, K)
        for i in range(N):
            for j in range(K):
                want[i, j] = w[i, j].float() * sf[i // b, j // b]
        assert torch.equal(dequant_blocked(w, s), want)


def test_v4_ue8m0_block32_checkpoint(tmp_path):
    """The V4 family's checkpoint format: e4m3 projections with 32 x 32 UE8M0
    block scales (float8_e8m0fnu `weight_scale_inv`).  The config round-trips
    and the engine built from the checkpoint generates exactly what a model
    built from the dequantized weights does."""
    from b200ds import EngineConfig, SamplingParams, build_model_from
    from b200ds.config import ModelConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.models.loader import load_checkpoint, save_checkpoint_fp8
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.ops.quant import dequant_blocked
    cfg = tiny_v4_config()
    save_checkpoint_fp8(init_weights_v4(cfg, 0), str(tmp_path), cfg, block=32, ue8m0=True)
    cfg2 = ModelConfig.from_hf(str(tmp_path / "config.json"))
    assert cfg2.is_v4 and cfg2.hc_mult == cfg.hc_mult and cfg2.engram_layers == cfg.engram_layers
    ck = load_checkpoint(str(tmp_path))
    s = ck["model.layers.0.self_attn.wqkv_a.weight_scale_inv"]
    assert s.dtype == torch.float8_e8m0fnu
    w = ck["model.layers.0.self_attn.wqkv_a.weight"]
    assert w.dtype == torch.float8_e4m3fn and s.shape == ((w.shape[0] + 31) // 32, (w.shape[1] + 31) // 32)
    deq = {k: (dequant_blocked(v, ck[k + "_scale_inv"]) if k + "_scale_inv" in ck else v)
           for k, v in ck.items() if not k.endswith("_scale_inv")}
    prompts = torch.randint(0, cfg.vocab_size, (2, 13), generator=torch.Generator().manual_seed(4)).tolist()
    outs = []
    for weights in (str(tmp_path), deq):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False)
        eng = Engine(build_model_from(cfg2, ecfg, weights, device="cpu"), ecfg)
        outs.append([o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=5))])
    assert outs[0] == outs[1]
