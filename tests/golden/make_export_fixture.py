"""Generate the int8-export fixture that pins mamba_integer_b200.export_format.

Runs the reference exporter itself, scripts/export_int8.py:export_model(),
on a small seeded model (d_model 64, 2 layers, vocab 256, d_state 16,
dt_rank 16, random norm gains).  The exporter reads a config file and a
checkpoint from paths it computes at import and moves the model to CUDA; for
this run its module globals CONFIG_PATH / CHECKPOINT_PATH / OUTPUT_BIN point
at temporary files and Module.cuda / torch.load(map_location="cuda") are
redirected to the CPU.  The reference model's CPU forward on seeded ids gives
the logits the loaded model must reproduce.  Writes

  export_tiny.bin    the exporter's output, committed (~185 KB);
  export_tiny.json   config, ids, sha256 of the logits and of every exported
                     array as the reference model holds it.

Only runs where the reference checkout exists; $MI_REFERENCE_ROOT (required)
names it:

    MI_REFERENCE_ROOT=<reference checkout> python tests/golden/make_export_fixture.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mamba_integer_b200 import synth  # noqa: E402

CONFIG = {"d_model": 64, "n_layer": 2, "vocab_size": 256, "ssm_cfg": {"d_state": 16, "dt_rank": 16}}
SEED = 21
IDS_SHAPE = (2, 24)


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def state_dict():
    sd = synth.model_state_dict(CONFIG, SEED)
    g = torch.Generator().manual_seed(SEED + 1)
    for k in list(sd):
        if k.endswith("norm.gamma") or k == "norm_f.gamma":
            sd[k] = 0.5 + torch.rand(sd[k].shape, generator=g)
    return sd


def ids():
    g = torch.Generator().manual_seed(SEED + 2)
    return torch.randint(0, CONFIG["vocab_size"], IDS_SHAPE, generator=g, dtype=torch.int64)


def main() -> None:
    ref_root = os.environ.get("MI_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("set MI_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, os.path.join(ref_root, "src"))
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import export_int8  # noqa: E402  (the reference exporter)
    import mamba_integer_model as ref_model  # noqa: E402

    sd = state_dict()
    out_bin = os.path.join(HERE, "export_tiny.bin")
    with tempfile.TemporaryDirectory() as tmp:
        cfg_path = os.path.join(tmp, "config.json")
        ckpt_path = os.path.join(tmp, "model.pt")
        with open(cfg_path, "w") as f:
            json.dump(CONFIG, f)
        torch.save(sd, ckpt_path)
        export_int8.CONFIG_PATH, export_int8.CHECKPOINT_PATH, export_int8.OUTPUT_BIN = cfg_path, ckpt_path, out_bin
        cuda, load = torch.nn.Module.cuda, torch.load
        torch.nn.Module.cuda = lambda self, *a, **k: self
        torch.load = lambda p, map_location=None, **k: load(p, map_location="cpu", **k)
        try:
            export_int8.export_model()
        finally:
            torch.nn.Module.cuda, torch.load = cuda, load

    m = ref_model.MambaIntegerModel(CONFIG)
    m.load_state_dict(sd)
    m.eval()
    x = ids()
    with torch.no_grad():
        logits = m(x).numpy()
    arrays = {"embedding": sha(m.embedding.weight.detach().numpy()), "norm_f.gamma": sha(m.norm_f.gamma.detach().numpy())}
    wq, s = m.lm_head.get_ternary_weights()
    arrays["lm_head"] = [sha(wq.numpy()), float(s)]
    for i, blk in enumerate(m.layers):
        for name in ("in_proj", "x_proj", "dt_proj", "out_proj"):
            wq, s = getattr(blk, name).get_ternary_weights()
            arrays[f"layers.{i}.{name}"] = [sha(wq.numpy()), float(s)]
        arrays[f"layers.{i}.conv1d.weight"] = sha(blk.conv1d.weight.detach().numpy())
        arrays[f"layers.{i}.base_decay_nums"] = sha(blk.base_decay_nums.detach().round().int().numpy())
    fx = {"config": CONFIG, "seed": SEED, "ids": x.tolist(), "logits_shape": list(logits.shape),
          "logits_sha256": sha(logits), "logits_sample": logits[0, -1, :8].tolist(), "arrays": arrays,
          "bin_bytes": os.path.getsize(out_bin)}
    with open(os.path.join(HERE, "export_tiny.json"), "w") as f:
        json.dump(fx, f, indent=1)
    print("wrote", out_bin, fx["bin_bytes"], "bytes")


if __name__ == "__main__":
    main()
