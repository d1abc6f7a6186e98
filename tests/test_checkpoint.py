"""llama2.c checkpoints (run.c layout): the header and size checks on CPU, and on a GPU a
model loaded from a checkpoint written with the oracle's weights decodes exactly like the
oracle (fp32 bar, identical greedy ids) and holds the file's weights bit for bit."""
import numpy as np
import pytest

import ammon_b200 as ab

CFG = dict(dim=128, layers=2, heads=4, kv_heads=2, head_dim=32, hidden=256, vocab=96, seq=48)


def write_llama2c(path, weights, cfg, shared=False):
    """Writes a llama2.c checkpoint: 7 int32 then the fp32 tensors in run.c order."""
    c = cfg
    head = c["dim"] // c["heads"]
    hdr = np.array([c["dim"], c["hidden"], c["layers"], c["heads"], c["kv_heads"],
                    c["vocab"] if shared else -c["vocab"], c["seq"]], np.int32)
    parts = [weights("embed", 0)]
    for name in ("rms_att", "wq", "wk", "wv", "wo", "rms_ffn", "w1", "w2", "w3"):
        parts += [weights(name, layer) for layer in range(c["layers"])]
    parts += [weights("rms_final", 0), np.zeros(c["seq"] * head, np.float32)]
    if not shared:
        parts.append(weights("wcls", 0))
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        for p in parts:
            f.write(np.ascontiguousarray(p, np.float32).tobytes())


def _random_weights(cfg, seed=1):
    rng = np.random.default_rng(seed)
    qd = cfg["heads"] * cfg["head_dim"]
    kvd = cfg["kv_heads"] * cfg["head_dim"]
    shapes = {"embed": (cfg["vocab"], cfg["dim"]), "wcls": (cfg["vocab"], cfg["dim"]),
              "rms_final": (cfg["dim"],), "rms_att": (cfg["dim"],), "rms_ffn": (cfg["dim"],),
              "wq": (qd, cfg["dim"]), "wk": (kvd, cfg["dim"]), "wv": (kvd, cfg["dim"]),
              "wo": (cfg["dim"], qd), "w1": (cfg["hidden"], cfg["dim"]),
              "w2": (cfg["dim"], cfg["hidden"]), "w3": (cfg["hidden"], cfg["dim"])}
    return lambda name, layer: rng.standard_normal(shapes[name]).astype(np.float32)


@pytest.mark.parametrize("shared", [False, True])
def test_llama2c_header_gives_the_model_shape(tmp_path, shared):
    path = str(tmp_path / "model.bin")
    write_llama2c(path, _random_weights(CFG), CFG, shared)
    cfg = ab.LlamaModel.llama2c_config(path, batch=3, dtype=ab.BF16, rope_theta=500000.0)
    for k, v in CFG.items():
        assert getattr(cfg, k) == v, k
    assert cfg.batch == 3 and cfg.dtype == ab.BF16 and cfg.rope_theta == 500000.0


def test_llama2c_size_and_header_are_checked(tmp_path):
    path = tmp_path / "model.bin"
    write_llama2c(str(path), _random_weights(CFG), CFG)
    data = path.read_bytes()
    (tmp_path / "short.bin").write_bytes(data[:-4])
    with pytest.raises(ab.ValidationError, match="bytes, the header's shapes need"):
        ab.LlamaModel.llama2c_config(str(tmp_path / "short.bin"))
    bad = np.frombuffer(data[:28], np.int32).copy()
    bad[3] = 5  # dim 128 is not a multiple of 5 heads
    (tmp_path / "bad.bin").write_bytes(bad.tobytes() + data[28:])
    with pytest.raises(ab.ValidationError, match="implausible header"):
        ab.LlamaModel.llama2c_config(str(tmp_path / "bad.bin"))
    with pytest.raises(ab.ValidationError, match="cannot open"):
        ab.LlamaModel.llama2c_config(str(tmp_path / "missing.bin"))


@pytest.mark.gpu
def test_llama2c_checkpoint_decodes_like_the_oracle(tmp_path, orc):
    o = orc.Model(**CFG, seed=19)
    path = str(tmp_path / "model.bin")
    write_llama2c(path, o.weight, CFG)
    rt = ab.create_runtime(0)
    m = ab.LlamaModel.from_llama2c(rt, path)
    for name in ("embed", "wcls", "rms_final"):
        assert np.array_equal(m.weight(name).read(), o.weight(name)), name
    for name in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn"):
        assert np.array_equal(m.weight(name, 1).read(), o.weight(name, 1)), name
    for pos, tok in enumerate([5, 90, 12, 12, 44, 3]):
        got = m.step(tok, pos)
        want = o.step(tok, pos)
        assert np.abs(got - want).max() / np.abs(want).max() < 1e-5, pos
        assert int(np.argmax(got)) == orc.sample_argmax(want)
    m.close()
    # a shared classifier is the embedding
    write_llama2c(path, o.weight, CFG, shared=True)
    m = ab.LlamaModel.from_llama2c(rt, path, dtype=ab.BF16)
    assert np.array_equal(m.weight("wcls").read(), m.weight("embed").read())
    assert np.array_equal(m.weight("embed").read(), orc.to_bf16_bits(o.weight("embed"))
                          .reshape(CFG["vocab"], CFG["dim"]))
    m.close()
    rt.close()
