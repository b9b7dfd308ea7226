"""Generate bench_c4_seq0.json: the oracle's logits for the first sequence of
bench.py's config-4 workload (24 layers, d_model 768, vocab 32768, 2048 tokens
of the seed-3 Zipf ids, the seed-3 synthetic weights), as sha256 hashes of the
last position's logits and of the full [2048, 32768] block, plus a few raw
values.

bench.py hashes the same rows of its own logits after the timed steps and
reports whether they match; tests/test_gpu_fullsize.py compares the full rows.
The oracle (oracle/, a C restatement pinned bit-for-bit to the reference's own
outputs by the other fixtures in this folder) computes them on the CPU:

    python tests/golden/make_bench_hash.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mamba_integer_b200 import synth  # noqa: E402
from oracle import model as om  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    c = synth.CONFIGS["c4"]
    cfg = synth.model_config("c4")
    sd = synth.model_state_dict(cfg, c["seed"])
    ids = synth.input_ids("c4", c["batch"], c["seq_len"])[:1].numpy()
    logits = om.forward(om.prepare(sd), cfg, ids, nthreads=os.cpu_count() or 1)[0]  # [2048, 32768]
    out = {
        "workload": "config4_prefill_24L_d768_b64x2048",
        "sequence": 0,
        "tokens": int(ids.shape[1]),
        "ids_sha256": sha(ids[0]),
        "last_logits_sha256": sha(logits[-1]),
        "logits_sha256": sha(logits),
        "last_logits_head": [float(v) for v in logits[-1, :8]],
        "source": "oracle/ (C restatement of the reference CPU path) on the CPU",
    }
    with open(os.path.join(HERE, "bench_c4_seq0.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
