"""Continuous-batching request loop over the slot engine, and a seeded synthetic multi-turn workload.

``run_requests`` follows the scheduling of the reference's driver loop (src/cb_run.py:254-378,
whole-prompt admission): while requests are pending and slots are free, every free slot takes the
next pending request and the admitted prompts go through packed ``prefill_batch`` calls; then one
``decode_step`` advances every active slot by one greedy token.  When a request has generated its
turn's tokens, its slot is freed; a multi-turn request then goes to the back of the queue with its
whole conversation as the next prompt (prompt + generated tokens + the next turn's appended
tokens), as the reference re-queues an agent request after a tool call (src/cb_run.py:197-225,
``finish``).

``synthetic_requests`` draws the BASELINE configs 3/4 workload: prompts of uniform random token
ids with lengths U[300, 700], 1-6 turns per request, each later turn appending U[50, 300] random
tokens, 512 greedy tokens per turn.  The reference ran agent datasets with real tokenizers and
weights; none of that is needed to exercise the engine, so token ids are drawn uniformly.

Every rank of a tensor-parallel engine runs the same loop on the same requests: the tokens are
identical on all ranks, so all ranks take the same scheduling decisions and collective steps.
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

import torch


@dataclass
class Request:
    rid: int
    turns: int                    # turns in total (1..6)
    prompt: torch.Tensor          # [L] int64 token ids of the current turn's prompt (host)
    appends: list                 # [turns - 1] tensors appended before each later turn
    turn: int = 0
    gen: list = field(default_factory=list)
    last: int = 0


def synthetic_requests(n, vocab, seed=0, prompt_len=(300, 700), max_turns=6, append_len=(50, 300)):
    """``n`` seeded multi-turn requests (length ranges inclusive, ids uniform in [0, vocab))."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for rid in range(n):
        L = int(torch.randint(prompt_len[0], prompt_len[1] + 1, (1,), generator=g))
        turns = int(torch.randint(1, max_turns + 1, (1,), generator=g))
        prompt = torch.randint(0, vocab, (L,), generator=g)
        appends = [torch.randint(0, vocab, (int(torch.randint(append_len[0], append_len[1] + 1, (1,), generator=g)),),
                                 generator=g) for _ in range(turns - 1)]
        out.append(Request(rid, turns, prompt, appends))
    return out


def max_context(reqs, gen_tokens):
    """Longest context any turn of ``reqs`` reaches (its final prompt + its generated tokens)."""
    return max(int(r.prompt.numel()) + sum(int(a.numel()) for a in r.appends) + r.turns * gen_tokens
               for r in reqs)


def run_requests(eng, reqs, gen_tokens=512, prefill_token_budget=32768, on_step=None):
    """Serve ``reqs`` (mutated) on ``eng`` until every turn of every request is done.

    Admitted prompts are prefilled in packed groups of at most ``prefill_token_budget`` tokens.
    ``on_step(kind, seconds, info)`` is called after each prefill / decode call with the wall time
    of the call (each call ends with the host read of its tokens, so the time covers its kernels).
    Returns the counts and times of the run."""
    pending = deque(reqs)
    free = list(range(eng.N))[::-1]
    slot_req = [None] * eng.N
    st = dict(prefill_calls=0, prefill_tokens=0, prefill_s=0.0, decode_steps=0, decode_tokens=0, decode_s=0.0,
              turns=0, requests=0, max_active=0)

    def finish(s):
        r = slot_req[s]
        slot_req[s] = None
        eng.free(s)
        free.append(s)
        st["turns"] += 1
        if r.turn + 1 < r.turns:            # next turn: the whole conversation is the new prompt
            r.prompt = torch.cat([r.prompt, torch.tensor(r.gen, dtype=torch.long), r.appends[r.turn]])
            r.turn += 1
            r.gen = []
            pending.append(r)
        else:
            st["requests"] += 1

    t_start = time.perf_counter()
    while pending or any(x is not None for x in slot_req):
        if free and pending:
            group = []
            while free and pending:
                group.append((pending.popleft(), free.pop()))
            i = 0
            while i < len(group):
                sub, tok = [], 0
                while i < len(group) and (not sub or tok + group[i][0].prompt.numel() <= prefill_token_budget):
                    sub.append(group[i])
                    tok += int(group[i][0].prompt.numel())
                    i += 1
                t0 = time.perf_counter()
                firsts = eng.prefill_batch([s for _, s in sub], [r.prompt[None] for r, _ in sub])
                dt = time.perf_counter() - t0
                st["prefill_calls"] += 1
                st["prefill_tokens"] += tok
                st["prefill_s"] += dt
                if on_step is not None:
                    on_step("prefill", dt, dict(tokens=tok, seqs=[int(r.prompt.numel()) for r, _ in sub]))
                for (r, s), f in zip(sub, firsts):
                    r.gen = [int(f)]
                    r.last = int(f)
                    slot_req[s] = r
                    if len(r.gen) >= gen_tokens:
                        finish(s)
        active = [s for s in range(eng.N) if slot_req[s] is not None]
        if not active:
            continue
        st["max_active"] = max(st["max_active"], len(active))
        ctx = [eng.lens[s] for s in active]
        t0 = time.perf_counter()
        nxt = eng.decode_step(active, [slot_req[s].last for s in active])
        dt = time.perf_counter() - t0
        st["decode_steps"] += 1
        st["decode_tokens"] += len(active)
        st["decode_s"] += dt
        if on_step is not None:
            on_step("decode", dt, dict(active=len(active), ctx=ctx))
        for s, t in zip(active, nxt):
            r = slot_req[s]
            r.gen.append(int(t))
            r.last = int(t)
            if len(r.gen) >= gen_tokens:
                finish(s)
    st["makespan_s"] = time.perf_counter() - t_start
    return st
