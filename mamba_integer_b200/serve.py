"""Continuous-batching greedy generation over the decode kernels.

The reference generates for one prompt at a time by recomputing the whole
forward per token (scripts/inference.py:148-160).  `DecodeServer` keeps a
fixed set of stream slots resident on the GPU (conv windows and scan states of
`slots` streams, see decode.StreamStates) and serves a queue of requests:

  * admission: queued requests take free slots; prompts of equal length are
    prefilled together by the prefill kernels, their final states are copied
    into their slots, and the argmax of their last-position logits is their
    first generated token;
  * step: one decode step (a replayed CUDA graph) advances every slot; each
    active request appends its slot's argmax;
  * retirement: a request finishes after `max_new_tokens` tokens or on
    `eos_id`; its slot is free for the next admission (stale state there is
    overwritten by the next prefill; idle slots are computed and ignored).

The host runs one step behind the GPU: a call launches step t (its next ids
stay on the device as step t+1's input and are copied to pinned host memory
behind an event), then reads step t-1's ids and does the bookkeeping while
step t runs.  A request that finished at step t-1 has had step t computed for
its slot too; that token is dropped (each slot's step is credited only to the
request that held the slot when the step was launched and still holds it).

Every request gets exactly the tokens greedy full-recompute generation gives
its prompt alone: streams never interact (every operation is per stream), so
neither the other slots nor the admission time change a stream's bits.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from .decode import DecodeEngine


@dataclass
class Request:
    rid: int
    prompt: List[int]
    max_new_tokens: int
    tokens: List[int] = field(default_factory=list)


class DecodeServer:
    def __init__(self, model, slots: int = 256, eos_id: Optional[int] = None,
                 engine: Optional[DecodeEngine] = None):
        self.eng = engine if engine is not None else DecodeEngine(model)
        self.eng.reserve(slots)
        self.n_slots = slots
        self.eos_id = eos_id
        self.active: List[Optional[Request]] = [None] * slots
        self.queue: deque = deque()
        self.finished: Dict[int, List[int]] = {}
        self._next_rid = 0
        self.steps = 0
        # two pinned buffers for the next ids of the last two launched steps, each
        # with the event its device-to-host copy completes; the launched step whose
        # ids are not read yet, with the slot owners at its launch
        # (an engine whose ids live on the host -- a stand-in for host tests -- needs neither)
        on_gpu = self.eng.ws.ids.is_cuda
        self._host_ids = [torch.empty(slots, dtype=torch.int64, pin_memory=on_gpu) for _ in range(2)]
        self._ready = [torch.cuda.Event() if on_gpu else None for _ in range(2)]
        self._inflight = None

    def submit(self, prompt: Sequence[int], max_new_tokens: int) -> int:
        if len(prompt) == 0 or max_new_tokens <= 0:
            raise ValueError("a request needs a non-empty prompt and max_new_tokens >= 1")
        rid = self._next_rid
        self._next_rid += 1
        self.queue.append(Request(rid, [int(t) for t in prompt], int(max_new_tokens)))
        return rid

    def pending(self) -> int:
        return len(self.queue) + sum(r is not None for r in self.active) + (self._inflight is not None)

    # -- internals -------------------------------------------------------------
    def _append(self, slot: int, tok: int) -> None:
        r = self.active[slot]
        r.tokens.append(tok)
        if len(r.tokens) >= r.max_new_tokens or (self.eos_id is not None and tok == self.eos_id):
            self.finished[r.rid] = r.tokens
            self.active[slot] = None

    def _admit(self) -> None:
        free = [i for i, r in enumerate(self.active) if r is None]
        while free and self.queue:
            # the next request and every queued request of the same prompt length
            L = len(self.queue[0].prompt)
            group = []
            for r in list(self.queue):
                if len(group) == len(free):
                    break
                if len(r.prompt) == L:
                    group.append(r)
            for r in group:
                self.queue.remove(r)
            slots = [free.pop(0) for _ in group]
            ids = torch.tensor([r.prompt for r in group], dtype=torch.int64)
            logits = self.eng.prefill_slots(slots, ids)
            first = self.eng.argmax(logits)
            self.eng.ws.ids.index_copy_(0, torch.as_tensor(slots, device=first.device), first)
            for s, r, tok in zip(slots, group, first.tolist()):
                self.active[s] = r
                self._append(s, tok)
            free = [i for i, r in enumerate(self.active) if r is None]

    def _consume(self, k: int, owners: List[Optional[Request]]) -> None:
        """Credit a launched step's ids (pinned buffer k) to the slots' owners at launch."""
        if self._ready[k] is not None:
            self._ready[k].synchronize()
        toks = self._host_ids[k].tolist()
        for s, r in enumerate(owners):
            if r is not None and self.active[s] is r:
                self._append(s, toks[s])

    # -- public loop -------------------------------------------------------------
    def step(self) -> bool:
        """Admit what fits, launch one decode step if any slot is active, then do the
        previous step's bookkeeping; False when nothing is left."""
        self._admit()
        launched = None
        if any(r is not None for r in self.active):
            ws = self.eng.ws
            self.eng.step(ws.ids)
            nxt = self.eng.next_ids()
            ws.ids.copy_(nxt)  # every slot's next input is its own last token
            k = self.steps & 1
            self._host_ids[k].copy_(nxt, non_blocking=self._ready[k] is not None)
            if self._ready[k] is not None:
                self._ready[k].record()
            launched = (k, list(self.active))
            self.steps += 1
        if self._inflight is not None:
            self._consume(*self._inflight)
        self._inflight = launched
        return self.pending() > 0

    def run(self) -> Dict[int, List[int]]:
        """Serve until every submitted request has finished."""
        while self.step():
            pass
        return self.finished
