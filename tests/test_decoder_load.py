"""Loading the decoder from a checkpoint directory and its INT8 overlay
(Model::load_with_quantization, src/model/mod.rs:81-105; ModelConfig::
from_json, src/model/config.rs:69-117; Decoder::new's shape checks,
src/decoder/mod.rs:32-83).

CPU tests: the configuration rules (the fields, defaults and rejections of
tests/config.rs and ModelConfig::from_json).  GPU tests: a synthetic
two-layer checkpoint (BF16 source, a dense layer and an MoE layer) and its
overlay are loaded; every device weight is checked against the source
(quantized by the oracle, or the source bits) and decode steps through the
loaded decoder are checked against the oracle's composition of the
reference operations."""
import json
import os
import struct

import numpy as np
import pytest

import oracle

BASE = {"model_type": "unlimited-ocr", "hidden_size": 256, "intermediate_size": 352,
        "moe_intermediate_size": 128, "num_hidden_layers": 2, "num_attention_heads": 2,
        "num_key_value_heads": 2, "n_routed_experts": 8, "n_shared_experts": 2,
        "num_experts_per_tok": 2, "first_k_dense_replace": 1, "use_mla": False,
        "vocab_size": 384, "sliding_window": 4}


def kind(fn):
    import uocr_q8
    with pytest.raises(uocr_q8.OcrError) as e:
        fn()
    return e.value.kind


def test_config_defaults_and_fields():
    from uocr_q8.decoder import config_from_json
    c = config_from_json(json.dumps(BASE))
    assert (c.hidden, c.heads, c.layers, c.first_dense, c.experts, c.top_k) == (256, 2, 2, 1, 8, 2)
    assert (c.expert_width, c.shared_width, c.dense_width, c.vocab) == (128, 256, 352, 384)
    assert (c.window, c.eps, c.theta, c.max_positions) == (4, 1e-6, 10000.0, 32768)
    assert (c.normalize, c.routed_scale, c.head_dim) == (False, 1.0, 128)
    d = dict(BASE)
    del d["sliding_window"]
    assert config_from_json(json.dumps(d)).window == 128


@pytest.mark.parametrize("change", [
    {"model_type": "other"}, {"use_mla": True}, {"attention_bias": True},
    {"rope_scaling": {"type": "linear"}}, {"topk_method": "noaux_tc"},
    {"scoring_func": "sigmoid"}, {"moe_layer_freq": 2}])
def test_config_unsupported(change):
    from uocr_q8.decoder import config_from_json
    assert kind(lambda: config_from_json(json.dumps({**BASE, **change}))) == "Unsupported"


@pytest.mark.parametrize("change", [
    {"hidden_size": 0}, {"num_attention_heads": 0}, {"hidden_size": 258},
    {"hidden_size": 6, "num_attention_heads": 2, "num_key_value_heads": 2},
    {"num_key_value_heads": 1}, {"num_hidden_layers": 0}, {"vocab_size": 0},
    {"intermediate_size": 0}, {"moe_intermediate_size": 0}, {"n_shared_experts": 0},
    {"num_experts_per_tok": 0}, {"num_experts_per_tok": 9}, {"first_k_dense_replace": 3},
    {"sliding_window": 0}, {"max_position_embeddings": 0}, {"rms_norm_eps": 0.0},
    {"rms_norm_eps": -1e-6}, {"rope_theta": 0.0}, {"routed_scaling_factor": 0.0}])
def test_config_shape_rejections(change):
    from uocr_q8.decoder import config_from_json
    assert kind(lambda: config_from_json(json.dumps({**BASE, **change}))) == "Shape"


def test_config_json_errors():
    from uocr_q8.decoder import config_from_json
    assert kind(lambda: config_from_json("{")) == "Json"
    d = dict(BASE)
    del d["vocab_size"]
    assert kind(lambda: config_from_json(json.dumps(d))) == "Json"


def test_dynamic_mode_needs_overlay(tmp_path):
    from uocr_q8 import QuantizationMode
    from uocr_q8.decoder import load_decoder
    assert kind(lambda: load_decoder(None, str(tmp_path), None,
                                     QuantizationMode.DYNAMIC_ACTIVATIONS)) == "Format"


# ---- GPU: a synthetic checkpoint and its overlay ------------------------------

def bf16_bits(rng, shape, scale):
    f = (rng.standard_normal(shape) * scale).astype(np.float32)
    return (f.view(np.uint32) >> 16).astype(np.uint16)


def bf16_float(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def write_checkpoint(d, seed=3):
    """config.json and model-00001-of-000001.safetensors (BF16 matrices,
    F32 norms) of the BASE configuration; returns name -> array (BF16 bit
    patterns as uint16, norms as float32)."""
    rng = np.random.default_rng(seed)
    H, F, E, W, S, V = 256, 352, 8, 128, 256, 384
    t = {"model.embed_tokens.weight": bf16_bits(rng, (V, H), 1.0),
         "model.norm.weight": (rng.random(H) * 0.5 + 0.75).astype(np.float32),
         "lm_head.weight": bf16_bits(rng, (V, H), 0.05)}
    for i in range(2):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = (rng.random(H) * 0.5 + 0.75).astype(np.float32)
        t[f"{p}.post_attention_layernorm.weight"] = (rng.random(H) * 0.5 + 0.75).astype(np.float32)
        for q in "qkvo":
            t[f"{p}.self_attn.{q}_proj.weight"] = bf16_bits(rng, (H, H), 0.05)
        ffns = [(f"{p}.mlp", F)] if i == 0 else \
            [(f"{p}.mlp.shared_experts", S)] + [(f"{p}.mlp.experts.{e}", W) for e in range(E)]
        for name, width in ffns:
            t[f"{name}.gate_proj.weight"] = bf16_bits(rng, (width, H), 0.05)
            t[f"{name}.up_proj.weight"] = bf16_bits(rng, (width, H), 0.05)
            t[f"{name}.down_proj.weight"] = bf16_bits(rng, (H, width), 0.05)
        if i == 1:
            t[f"{p}.mlp.gate.weight"] = bf16_bits(rng, (E, H), 0.05)
    header, data, off = {}, bytearray(), 0
    for name in sorted(t):
        a = t[name]
        dt = "BF16" if a.dtype == np.uint16 else "F32"
        b = a.astype("<u2" if dt == "BF16" else "<f4").tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        data += b
        off += len(b)
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((-len(raw)) % 8)
    with open(os.path.join(d, "model-00001-of-000001.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(raw)) + raw + bytes(data))
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(BASE, f)
    return t


def to_f32(a):
    return bf16_float(a) if a.dtype == np.uint16 else a


@pytest.fixture(scope="module")
def loaded(tmp_path_factory, request):
    import uocr_q8
    from uocr_q8.decoder import load_decoder
    from uocr_q8.overlay import write_overlay
    ctx = request.getfixturevalue("ctx")
    d = str(tmp_path_factory.mktemp("ckpt"))
    t = write_checkpoint(d)
    ov = os.path.join(d, "q8.safetensors")
    write_overlay(os.path.join(d, "model-00001-of-000001.safetensors"), ov, ctx)
    return ctx, d, ov, t, load_decoder(ctx, d, ov, uocr_q8.QuantizationMode.WEIGHTS_ONLY)


def same_q8(m, w, s):
    """Device matrix m equals the q8 pair (w, s), bit for bit."""
    dw, ds = m.download()
    return np.array_equal(dw, w) and np.array_equal(ds.view(np.uint32), s.view(np.uint32))


@pytest.mark.gpu
def test_loaded_weights_are_the_source(loaded):
    import torch
    _, _, _, t, dec = loaded
    host = lambda x: x.detach().cpu().numpy()  # noqa: E731
    q = lambda name: oracle.quantize(to_f32(t[name]))  # noqa: E731
    for i, L in enumerate(dec.layers):
        p = f"model.layers.{i}"
        parts = [q(f"{p}.self_attn.{c}_proj.weight") for c in "qkv"]
        assert same_q8(L.qkv, np.concatenate([m.w for m in parts]),
                       np.concatenate([m.s for m in parts]))
        o = q(f"{p}.self_attn.o_proj.weight")
        assert same_q8(L.o, o.w, o.s)
        assert np.array_equal(host(L.input_norm), t[f"{p}.input_layernorm.weight"])
        assert np.array_equal(host(L.post_norm), t[f"{p}.post_attention_layernorm.weight"])
        if i == 0:
            assert L.moe is None and L.dense_width == 352
            g, u, dn = (q(f"{p}.mlp.{c}_proj.weight") for c in ("gate", "up", "down"))
            for m, ref in ((L.dense[0], g), (L.dense[1], u)):
                assert (m.rows, m.cols) == (384, 256)
                assert same_q8(m, np.concatenate([ref.w, np.zeros((32, 256), np.int8)]),
                               np.concatenate([ref.s, np.zeros((32, 8), np.float32)]))
            assert (L.dense[2].rows, L.dense[2].cols) == (256, 384)
            assert same_q8(L.dense[2], np.concatenate([dn.w, np.zeros((256, 32), np.int8)], 1),
                           np.concatenate([dn.s, np.zeros((256, 1), np.float32)], 1))
        else:
            assert np.array_equal(host(L.router.view(torch.int16)).view(np.uint16),
                                  t[f"{p}.mlp.gate.weight"])
            shared, experts = L.moe._keep
            names = [f"{p}.mlp.shared_experts"] + [f"{p}.mlp.experts.{e}" for e in range(8)]
            for mats, name in zip([shared] + experts, names):
                for m, c in zip(mats, ("gate", "up", "down")):
                    ref = q(f"{name}.{c}_proj.weight")
                    assert same_q8(m, ref.w, ref.s)
    assert np.array_equal(host(dec.embedding.view(torch.int16)).view(np.uint16),
                          t["model.embed_tokens.weight"])
    assert np.array_equal(host(dec.final_norm), t["model.norm.weight"])
    head = q("lm_head.weight")
    assert same_q8(dec.lm_head, head.w, head.s)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 2])
def test_loaded_decoder_steps_match_oracle(loaded, mode):
    from test_gpu_decoder import dev, host, host_decoder, oracle_step
    from uocr_q8.decoder import DecodeState, decode_step
    ctx, _, _, _, dec = loaded
    cfg = dec.cfg
    layers, emb, final_norm, head = host_decoder(dec)
    batch, prefix = 2, 2
    state = DecodeState(dec, batch, prefix)
    rng = np.random.default_rng(11 + mode)
    caches = []
    for b in range(batch):  # a prompt prefix of random keys and values
        seq = []
        for cache in state.caches:
            k, v = (rng.standard_normal((prefix, cfg.hidden)).astype(np.float32) for _ in "kv")
            cache.prefill(b, dev(k), dev(v))
            c = oracle.LayerCache(cfg.heads, cfg.head_dim, cfg.window)
            c.prefill(k, v, prefix)
            seq.append(c)
        caches.append(seq)
    for step in range(6):  # the 4-token window wraps
        tokens = rng.integers(0, cfg.vocab, batch)
        logits = host(decode_step(dec, state, dev(tokens.astype(np.int64)), mode))
        ctx.sync()
        for b in range(batch):
            ref = oracle_step(cfg, layers, emb, final_norm, head, caches[b], int(tokens[b]), mode)
            scale = float(np.max(np.abs(ref)))
            err = float(np.max(np.abs(logits[b].astype(np.float64) - ref)))
            assert err <= (1e-3 if mode == 0 else 1e-2) * scale, (step, b, err, scale)
    state.free()


@pytest.mark.gpu
def test_load_rejects_shape_and_missing_overlay(loaded, tmp_path):
    import uocr_q8
    from uocr_q8.decoder import load_decoder
    ctx, d, ov, _, _ = loaded
    assert kind(lambda: load_decoder(ctx, d, None)) == "Unsupported"
    # a configuration whose dense width disagrees with the checkpoint
    bad = tmp_path / "bad"
    bad.mkdir()
    for f in ("model-00001-of-000001.safetensors",):
        os.link(os.path.join(d, f), str(bad / f))
    (bad / "config.json").write_text(json.dumps({**BASE, "intermediate_size": 320}))
    assert kind(lambda: load_decoder(ctx, str(bad), ov,
                                     uocr_q8.QuantizationMode.WEIGHTS_ONLY)) == "Shape"
