"""Checkpoint format: config parsing (src/config.rs:43-66) and the safetensors round trip."""
import numpy as np

from conftest import pkg

cfgm = pkg("config")
W = pkg("weights")


def test_layer_dims_and_types(model_dir):
    c = cfgm.ModelConfig.load(model_dir).text
    assert c.num_hidden_layers == 24
    glob = [i for i in range(24) if not c.is_sliding(i)]
    assert glob == [5, 11, 17, 23]
    assert c.layer_dims(0) == (256, 2) and c.layer_dims(5) == (512, 1)
    assert c.rope_theta(0) == 1e4 and c.rope_theta(5) == 1e6


def test_checkpoint_tensors(model_dir):
    st = W.SafeTensors(model_dir / "model.safetensors")
    assert st.f32("language_model.layers.5.self_attn.q_proj.weight").shape == (2048, 512)
    assert st.f32("language_model.layers.0.self_attn.k_proj.weight").shape == (512, 512)
    assert st.scalar("language_model.layers.3.layer_scalar") == 1.0
    np.testing.assert_array_equal(st.f32("language_model.norm.weight"), np.ones(512, np.float32))
    qn = st.f32("language_model.layers.0.self_attn.q_norm.weight")
    assert np.all(qn == np.float32(0.25))
    w = st.f32("language_model.ple.per_layer_model_projection.weight")
    assert w.shape == (12288, 512) and abs(float(w.std()) - 0.02) < 1e-3


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-8, 3.0e38], dtype=np.float32)
    r = W.bf16_round(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.015625)
    assert np.all(W.bf16_bits_to_f32(W.f32_to_bf16_bits(r)) == r)


def test_deterministic_generation(tmp_path):
    cfg = cfgm.synthetic_config(num_hidden_layers=2, vision_layers=1)
    cfg["text_config"]["vocab_size"] = 64
    cfg["vision_config"]["position_embedding_size"] = 16
    a = W.make_random_checkpoint(tmp_path / "a", seed=5, cfg=cfg)
    b = W.make_random_checkpoint(tmp_path / "b", seed=5, cfg=cfg)
    assert a.read_bytes() == b.read_bytes()
