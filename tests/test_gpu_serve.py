"""Continuous-batching generation: every request must get the tokens greedy
full-recompute generation gives its prompt alone (the reference's loop,
scripts/inference.py:148-160, with argmax instead of sampling), whatever
shares the slots with it and whenever it is admitted."""
import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu


def _oracle_greedy(p, cfg, prompt, n_new, eos=None):
    from oracle import model as om
    seq = np.asarray(prompt, np.int64)[None, :]
    out = []
    for _ in range(n_new):
        tok = int(np.argmax(om.forward(p, cfg, seq)[0, -1]))
        out.append(tok)
        if eos is not None and tok == eos:
            break
        seq = np.concatenate([seq, [[tok]]], axis=1)
    return out


@pytest.mark.parametrize("use_graph", [True, False])
def test_server_requests_match_per_prompt_greedy_generation(cuda_dev, use_graph):
    from mamba_integer_b200.decode import DecodeEngine
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    from mamba_integer_b200.serve import DecodeServer
    from oracle import model as om
    cfg, sd, _ = cases.model_inputs("c1")
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    m = m.to(cuda_dev).eval()
    g = torch.Generator().manual_seed(11)
    lens, news = [5, 9, 5, 12, 3, 7, 5], [4, 6, 3, 5, 1, 2, 4]
    prompts = [torch.randint(0, cfg["vocab_size"], (n,), generator=g).tolist() for n in lens]
    srv = DecodeServer(m, slots=3, engine=DecodeEngine(m, use_graph=use_graph))
    rids = [srv.submit(pr, k) for pr, k in zip(prompts[:5], news[:5])]
    srv.step()
    srv.step()
    rids += [srv.submit(pr, k) for pr, k in zip(prompts[5:], news[5:])]  # arrive mid-flight
    out = srv.run()
    assert sorted(out) == sorted(rids)
    p = om.prepare(sd)
    for rid, pr, k in zip(rids, prompts, news):
        assert out[rid] == _oracle_greedy(p, cfg, pr, k), f"request {rid}"


def test_server_stops_at_eos(cuda_dev):
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    from mamba_integer_b200.serve import DecodeServer
    from oracle import model as om
    cfg, sd, _ = cases.model_inputs("c1")
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    m = m.to(cuda_dev).eval()
    p = om.prepare(sd)
    prompt = [3, 1, 4, 1, 5, 9]
    free_run = _oracle_greedy(p, cfg, prompt, 6)
    eos = free_run[2]  # stop at the third generated token
    srv = DecodeServer(m, slots=2, eos_id=eos)
    rid = srv.submit(prompt, 6)
    out = srv.run()
    assert out[rid] == free_run[: free_run.index(eos) + 1]
