"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the UNMODIFIED reference CPU path (imported from the reference checkout
named by $MI_REFERENCE_SRC, its src/ directory; required) on seeded inputs and
writes

  model_<case>.json   sha256 of every hooked stage output and of the logits of
                      MambaIntegerModel.forward, plus a few raw logit values;
  stages.npz          small stage-level input/output pairs with edge values
                      (quantisation ties, zero rows, huge/tiny values, every
                      power-of-2 threshold band, clamp edges, scan edge decays).

Inputs are regenerated from seeds by tests/golden/cases.py, so only outputs
are stored.  The fixtures are committed; this script is only needed to
regenerate them and only runs where the reference checkout exists.

    MI_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import cases  # noqa: E402


def sha(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


def _import_reference():
    src = os.environ.get("MI_REFERENCE_SRC")
    if not src:
        raise SystemExit("set MI_REFERENCE_SRC to the reference checkout's src/ directory")
    sys.path.insert(0, src)
    import mamba_integer_model as ref_model  # noqa: E402
    import rational_bitnet as ref_bitnet  # noqa: E402

    return ref_model, ref_bitnet


def model_case(ref_model, name: str):
    spec = cases.MODEL_CASES[name]
    cfg, sd, ids = cases.model_inputs(name)
    m = ref_model.MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    m.eval()
    caps = {}
    hooks = []
    for mod_name, mod in m.named_modules():
        key = cases.hook_key(mod_name)
        if key is None:
            continue

        def hook(mo, inp, out, key=key):
            caps[key] = out.detach().clone()

        hooks.append(mod.register_forward_hook(hook))
    with torch.no_grad():
        logits = m(ids).numpy()
    for h in hooks:
        h.remove()
    L = ids.shape[1]
    stage = {}
    for k, v in caps.items():
        if k.endswith("conv"):
            v = v.transpose(1, 2)[:, :L]  # conv1d output [B, C, L+3] -> [B, L, C]
        a = v.contiguous().numpy()
        stage[k] = sha(a.reshape(-1, a.shape[-1]))
    return {
        "case": name,
        "spec": spec,
        "logits_shape": list(logits.shape),
        "logits_sha256": sha(logits),
        "logits_sample": [float(x) for x in logits.reshape(-1)[:8]] + [float(x) for x in logits.reshape(-1)[-8:]],
        "stages_sha256": stage,
    }


def stage_fixtures(ref_model, ref_bitnet):
    out = {}
    with torch.no_grad():
        # activation quantisation
        xq_in = cases.quant_inputs()
        q, s = ref_bitnet.activation_quant_dynamic(torch.from_numpy(xq_in))
        out["quant.xq"] = q.numpy().astype(np.int8)
        out["quant.scale"] = s.numpy().reshape(-1)
        # squareplus(ste_clamp(x, -50, 50)) and ste_clamp on edge values
        e = torch.from_numpy(cases.edge_values())
        out["sqp.y"] = ref_model._squareplus_rational(ref_model.ste_clamp(e, -50.0, 50.0), num_iters=3).numpy()
        out["ste20.y"] = ref_model.ste_clamp(e, -20.0, 20.0).numpy()
        out["ste_dec.y"] = ref_model.ste_clamp(e, 0, 32000).numpy()
        dtv = ref_model.ste_clamp(ref_model._squareplus_rational(ref_model.ste_clamp(e, -20.0, 20.0), num_iters=3)
                                  * 0.01, 0.001, 0.1)
        out["dtv.y"] = dtv.numpy()
        # gate
        gy, gz = cases.gate_inputs()
        out["gate.y"] = (torch.from_numpy(gy) * ref_model._sigmoid_algebraic(torch.from_numpy(gz))).numpy()
        # BitShiftNorm (both centerings) across all threshold bands, random gamma / step
        nx, ng, nst = cases.norm_inputs()
        norm = ref_model.BitShiftNorm(nx.shape[-1])
        norm.gamma.copy_(torch.from_numpy(ng))
        norm.step_size.copy_(torch.from_numpy(nst))
        out["norm.y"] = norm(torch.from_numpy(nx)).numpy()
        var = torch.from_numpy(nx)
        var = var - var.mean(dim=-1, keepdim=True)
        var = var - var.mean(dim=-1, keepdim=True)
        out["norm.inv_rms"] = ref_model._find_power_of_2_scale(var.pow(2).mean(dim=-1, keepdim=True)).numpy().reshape(-1)
        # DyadicScanFunction CPU branch
        u, nums = cases.scan_inputs()
        shifts = torch.full_like(torch.from_numpy(nums), 15.0)
        out["scan.h"] = ref_model.DyadicScanFunction.apply(torch.from_numpy(u), torch.from_numpy(nums), shifts).numpy()
        # weight quantisation of a non-power-of-2 weight matrix
        w = cases.weight_input()
        wq, ws = ref_bitnet.weight_quant_ternary(torch.from_numpy(w))
        out["wq.q"] = wq.numpy().astype(np.int8)
        out["wq.scale"] = np.array([ws.item()], np.float32)
    return out


def main():
    ref_model, ref_bitnet = _import_reference()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in cases.MODEL_CASES:
        fx = model_case(ref_model, name)
        with open(os.path.join(HERE, f"model_{name}.json"), "w") as f:
            json.dump(fx, f, indent=1, sort_keys=True)
        print("wrote", name, fx["logits_sha256"][:16])
    st = stage_fixtures(ref_model, ref_bitnet)
    np.savez_compressed(os.path.join(HERE, "stages.npz"), **st)
    print("wrote stages.npz", sorted(st))


if __name__ == "__main__":
    main()
