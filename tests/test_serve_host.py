"""DecodeServer's slot management on the CPU, with a stand-in engine whose
"model" is a toy rule: the first token of a prompt is sum(prompt) % V and
every next token is (previous + 1) % V.  Checks admission (equal-length
grouping, queueing beyond the slots), per-slot inputs, retirement and EOS."""
import torch

from mamba_integer_b200.serve import DecodeServer

V = 50


class FakeEngine:
    def __init__(self):
        self.prefill_calls = []

    def reserve(self, batch):
        self.ws = type("WS", (), {})()
        self.ws.ids = torch.zeros(batch, dtype=torch.int64)
        self._next = torch.zeros(batch, dtype=torch.int64)

    def prefill_slots(self, slots, prompt_ids):
        self.prefill_calls.append((list(slots), prompt_ids.shape[1]))
        logits = torch.zeros(prompt_ids.shape[0], V)
        logits[torch.arange(prompt_ids.shape[0]), prompt_ids.sum(1) % V] = 1.0
        return logits

    @staticmethod
    def argmax(logits):
        return torch.argmax(logits, dim=-1)

    def step(self, ids):
        self.ws.ids.copy_(ids)
        self._next = (self.ws.ids + 1) % V

    def next_ids(self):
        return self._next


def expected(prompt, n, eos=None):
    out, tok = [], sum(prompt) % V
    for _ in range(n):
        out.append(tok)
        if tok == eos:
            break
        tok = (tok + 1) % V
    return out


def test_slots_queueing_and_per_request_tokens():
    eng = FakeEngine()
    srv = DecodeServer(None, slots=2, engine=eng)
    reqs = [([1, 2, 3], 4), ([4, 5, 6], 2), ([7, 8], 5), ([9, 9, 9], 1), ([1], 3)]
    rids = [srv.submit(p, n) for p, n in reqs]
    out = srv.run()
    for rid, (p, n) in zip(rids, reqs):
        assert out[rid] == expected(p, n), rid
    # the first admission took both equal-length prompts together
    assert eng.prefill_calls[0] == ([0, 1], 3)
    assert all(r is None for r in srv.active) and not srv.queue


def test_eos_and_late_arrivals():
    eng = FakeEngine()
    srv = DecodeServer(None, slots=3, eos_id=12, engine=eng)
    a = srv.submit([10], 8)        # 10, 11, 12 -> stops at eos
    srv.step()
    b = srv.submit([3, 3], 3)      # arrives while a is running
    out = srv.run()
    assert out[a] == [10, 11, 12]
    assert out[b] == expected([3, 3], 3, eos=12)
