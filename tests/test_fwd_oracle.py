"""The whole-forward oracle (oracle/fwd_oracle.py) against the reference
engine's own logits (tests/golden/forward.npz, from tg_forward of
src/tgai_engine.c on the seeded models of tests/fwd_model.py).  CPU only."""
import os
import struct

import numpy as np
import pytest

import fwd_model as FM
import fwd_oracle
from conftest import GOLDEN


@pytest.mark.parametrize("name", sorted(FM.CONFIGS))
def test_oracle_reproduces_engine_logits(name):
    cfg = FM.CONFIGS[name]
    z = np.load(os.path.join(GOLDEN, "forward.npz"))
    assert int(z[f"{name}_seed"]) == FM.SEEDS[name]
    gold = z[f"{name}_logits"]
    o = fwd_oracle.Forward(cfg, FM.weights(cfg, FM.SEEDS[name]))
    steps = FM.script(cfg, FM.SEEDS[name])
    assert len(steps) == gold.shape[0]
    for i, (key, ids, pos) in enumerate(steps):
        lg = o.forward(key, ids, pos)
        err = np.abs(lg - gold[i]).max() / np.abs(gold[i]).max()
        assert err < 1e-6, (name, i, err)


def test_tg_writer_layout(tmp_path):
    cfg = FM.CONFIGS["dense"]
    w = {"token_embedding.weight": np.arange(12, dtype=np.float32).reshape(3, 4),
         "final_norm.weight": np.ones(4, np.float32)}
    path = tmp_path / "t.TG"
    FM.write_tg(str(path), cfg, w)
    raw = path.read_bytes()
    h = struct.unpack("<16I6Q4I", raw[:128])
    assert h[0] == 0x49414754 and h[1] == 1
    table_off, count, data_off = h[18], h[19], h[20]
    assert table_off == 128 and count == 2 and data_off % 64 == 0
    e = struct.unpack("<QQQII4II", raw[table_off:table_off + 52])
    assert e[0] == FM.fnv1a64("token_embedding.weight")
    assert e[4] == 2 and e[5:7] == (3, 4)
    got = np.frombuffer(raw[data_off + e[1]:data_off + e[1] + e[2]], np.float32)
    assert np.array_equal(got, np.arange(12, dtype=np.float32))
    # FNV-1a 64 of the empty string is the offset basis
    assert FM.fnv1a64("") == 0xcbf29ce484222325
