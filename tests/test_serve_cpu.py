"""CPU tests of the continuous-batching request loop (serve.run_requests) with a fake engine.

The loop must follow the reference driver's scheduling (src/cb_run.py:254-378): free slots admit
pending requests in packed prefills, every active slot decodes one token per step, a finished turn
frees its slot and a multi-turn request goes to the back of the queue with its whole conversation
(prompt + generated tokens + the next appended tokens) as the next prompt.
"""
import torch

from conftest import pkg


class FakeEngine:
    """Records calls; emits token = slot * 1000 + step so generated ids are traceable."""

    def __init__(self, n):
        self.N = n
        self.lens = [0] * n
        self.prefills = []
        self.steps = 0
        self.busy = set()

    def prefill_batch(self, slots, ids):
        for s, x in zip(slots, ids):
            assert s not in self.busy, "a slot was admitted twice"
            self.busy.add(s)
            self.lens[s] = int(x.numel())
        self.prefills.append([(s, x.reshape(-1).clone()) for s, x in zip(slots, ids)])
        return [7] * len(slots)

    def decode_step(self, slots, tokens):
        assert set(slots) <= self.busy
        self.steps += 1
        for s in slots:
            self.lens[s] += 1
        return [s * 1000 + self.steps for s in slots]

    def free(self, s):
        self.busy.discard(s)
        self.lens[s] = 0


def test_requests_complete_every_turn_with_growing_prompts():
    serve = pkg("serve")
    reqs = serve.synthetic_requests(7, vocab=50, seed=3, prompt_len=(5, 9), max_turns=3, append_len=(2, 4))
    first_prompts = {r.rid: r.prompt.clone() for r in reqs}
    eng = FakeEngine(3)
    seen = []
    st = serve.run_requests(eng, reqs, gen_tokens=4, on_step=lambda k, dt, info: seen.append(k))
    assert st["requests"] == 7 and st["turns"] == sum(r.turns for r in reqs)
    assert all(r.turn == r.turns - 1 for r in reqs)
    assert st["decode_tokens"] == 3 * st["turns"]          # the prefill gives the first of 4 tokens
    assert st["prefill_tokens"] == sum(x.numel() for call in eng.prefills for _, x in call)
    assert seen.count("decode") == st["decode_steps"] == eng.steps
    assert st["max_active"] <= 3 and not eng.busy
    # every later-turn prompt is the previous prompt + its 4 generated tokens + the appended tokens
    by_req = {}
    for call in eng.prefills:
        for s, x in call:
            rid = next(r.rid for r in reqs if torch.equal(x[:len(first_prompts[r.rid])], first_prompts[r.rid]))
            by_req.setdefault(rid, []).append(x)
    for r in reqs:
        ps = by_req[r.rid]
        assert len(ps) == r.turns
        for t in range(1, r.turns):
            prev, cur = ps[t - 1], ps[t]
            assert torch.equal(cur[:prev.numel()], prev)
            assert cur.numel() == prev.numel() + 4 + r.appends[t - 1].numel()
            assert torch.equal(cur[-r.appends[t - 1].numel():], r.appends[t - 1])
            assert cur[prev.numel()] == 7                    # the prefill's first token opens the turn


def test_admission_is_fifo_and_requeues_at_the_back():
    serve = pkg("serve")
    reqs = serve.synthetic_requests(4, vocab=50, seed=1, prompt_len=(3, 3), max_turns=1)
    reqs[0].turns, reqs[0].appends = 2, [torch.tensor([1, 2])]
    eng = FakeEngine(2)
    serve.run_requests(eng, reqs, gen_tokens=2)
    order = [x.numel() for call in eng.prefills for _, x in call]
    # requests 0 and 1 first, then 2 and 3 as they free up, then request 0's second turn (3 + 2 + 2)
    assert order[:4] == [3, 3, 3, 3] and order[4] == 7


def test_prefill_groups_respect_the_token_budget():
    serve = pkg("serve")
    reqs = serve.synthetic_requests(6, vocab=50, seed=2, prompt_len=(10, 10), max_turns=1)
    eng = FakeEngine(6)
    st = serve.run_requests(eng, reqs, gen_tokens=1, prefill_token_budget=25)
    assert [len(c) for c in eng.prefills] == [2, 2, 2] and st["prefill_calls"] == 3


def test_synthetic_workload_shapes():
    serve = pkg("serve")
    reqs = serve.synthetic_requests(200, vocab=248320, seed=0)
    assert all(300 <= r.prompt.numel() <= 700 for r in reqs)
    assert all(1 <= r.turns <= 6 and len(r.appends) == r.turns - 1 for r in reqs)
    assert all(50 <= a.numel() <= 300 for r in reqs for a in r.appends)
    assert {r.turns for r in reqs} == set(range(1, 7))
    assert serve.max_context(reqs, 512) <= 700 + 5 * 300 + 6 * 512
