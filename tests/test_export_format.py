"""The reference's int8 export format (scripts/export_int8.py:52-135), on the CPU.

tests/golden/export_tiny.bin was written by the reference exporter itself
(tests/golden/make_export_fixture.py); export_tiny.json holds hashes of the
reference model's arrays and logits.  Checked here: parsing, the model the
export describes (the oracle run from the parsed arrays reproduces the
reference logits bit for bit), and that loading and re-writing gives the same
bytes."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import model as om

GOLD = os.path.join(os.path.dirname(__file__), "golden")
BIN = os.path.join(GOLD, "export_tiny.bin")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def fx():
    with open(os.path.join(GOLD, "export_tiny.json")) as f:
        return json.load(f)


def test_parse_matches_reference_arrays(fx):
    from mamba_integer_b200.export_format import read_export
    e = read_export(BIN)
    assert e.config() == fx["config"]
    a = fx["arrays"]
    assert sha(e.embedding) == a["embedding"]
    assert sha(e.norm_f_gamma) == a["norm_f.gamma"]
    assert [sha(e.lm_head[1]), float(e.lm_head[0])] == a["lm_head"]
    for i, L in enumerate(e.layers):
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            s, w = getattr(L, name)
            assert [sha(w), float(s)] == a[f"layers.{i}.{name}"], (i, name)
        assert sha(L.conv_w) == a[f"layers.{i}.conv1d.weight"]
        assert sha(L.nums) == a[f"layers.{i}.base_decay_nums"]
        assert (L.shifts == 15).all() and (L.dt_bias == 0).all()


def test_oracle_on_exported_arrays_reproduces_reference_logits(fx):
    from mamba_integer_b200.export_format import read_export
    e = read_export(BIN)
    p = {"embedding.weight": e.embedding, "norm_f.gamma": e.norm_f_gamma,
         "norm_f.step_size": np.ones(1, np.float32), "lm_head.weight": (e.lm_head[1], e.lm_head[0])}
    for i, L in enumerate(e.layers):
        q = f"layers.{i}."
        p[q + "norm.gamma"], p[q + "norm.step_size"] = L.gamma, np.ones(1, np.float32)
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            s, w = getattr(L, name)
            p[q + name + ".weight"] = (w, s)
        p[q + "conv1d.weight"], p[q + "conv1d.bias"] = L.conv_w, L.conv_b
        p[q + "base_decay_nums"] = L.nums.astype(np.float32)
        p[q + "decay_shifts"] = L.shifts.astype(np.float32)
        p[q + "res_gate"] = L.res_gate
    logits = om.forward(p, e.config(), np.array(fx["ids"], np.int64))
    assert list(logits.shape) == fx["logits_shape"]
    assert sha(logits) == fx["logits_sha256"]


def test_load_then_write_gives_the_same_bytes(tmp_path):
    from mamba_integer_b200.export_format import load_export, write_export
    m = load_export(BIN)
    out = tmp_path / "again.bin"
    write_export(m, str(out))
    assert out.read_bytes() == open(BIN, "rb").read()


def test_rejects_bad_magic_and_truncation(tmp_path):
    from mamba_integer_b200.export_format import read_export
    data = open(BIN, "rb").read()
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"\x00\x00\x00\x00" + data[4:])
    with pytest.raises(ValueError, match="magic"):
        read_export(str(bad))
    short = tmp_path / "short.bin"
    short.write_bytes(data[:-10])
    with pytest.raises(ValueError, match="truncated"):
        read_export(str(short))
