"""GPU tests of the B200 engine against the reference's CBEngine on a tiny Qwen3.5.

The golden file (tests/golden/engine_tiny.npz) holds the weights of a tiny 3:1 GDN/attention
model and what the reference's CBEngine (src/cb_engine.py:80-355) produced on the CPU with its
own GDN plug-ins: two prompts prefilled into slots 1 and 0, then five dense decode steps.  The
engine here must reproduce the per-step logits (teacher-forced on the reference's tokens, so a
near-tie cannot send the two down different paths) and the GDN slot states, within bf16
tolerance; its own modes (CUDA-graph decode, packed prefill, chunked prefill, held slots) are
checked against each other.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, pkg

pytestmark = pytest.mark.gpu

DEV = "cuda"


def tiny_model():
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForConditionalGeneration
    from golden.make_golden import ENGINE_TEXT_CONFIG, ENGINE_VISION_CONFIG
    d = load_golden("engine_tiny.npz")
    cfg = Qwen3_5Config(text_config=ENGINE_TEXT_CONFIG, vision_config=ENGINE_VISION_CONFIG)
    model = Qwen3_5ForConditionalGeneration(cfg).to(torch.bfloat16)
    sd = {k[3:]: torch.from_numpy(np.ascontiguousarray(v)).to(torch.bfloat16) for k, v in d.items()
          if k.startswith("w::")}
    model.load_state_dict(sd, strict=True)
    return model.to(DEV).eval(), d


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    import sys, os
    sys.path.insert(0, os.path.join(os.path.dirname(__file__)))
    return tiny_model()


def _engine(model, graph=False, n_slots=2):
    eng_mod = pkg("engine")
    return eng_mod.CBEngine(model, n_slots=n_slots, t_max=128, device=DEV, graph_decode=graph)


def _logit_hook(model, store):
    return model.lm_head.register_forward_hook(lambda m, i, o: store.append(o.detach().float().cpu()))


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max()), bool(np.abs(a - b).max() <= atol + rtol * np.abs(b).max())


def test_engine_matches_reference_cbengine(setup):
    model, d = setup
    eng = _engine(model)
    logits = []
    h = _logit_hook(model, logits)
    ids_a = torch.tensor(d["ids_a"], dtype=torch.long, device=DEV)[None]
    ids_b = torch.tensor(d["ids_b"], dtype=torch.long, device=DEV)[None]
    eng.prefill(1, ids_a)
    eng.prefill(0, ids_b)
    pre = torch.stack([logits[0][0], logits[1][0]]).numpy()
    err, ok = _close(pre, d["pre_logits"], rtol=0, atol=0.15)
    assert ok, f"prefill logits differ by {err}"
    layers = [int(i) for i in d["gdn_layers"]]
    for j, i in enumerate(layers):
        err, ok = _close(eng.rec[i][:2].cpu(), d["rec_pre"][j])
        assert ok, f"layer {i} recurrent state after prefill differs by {err}"
        err, ok = _close(eng.conv[i][:2].float().cpu(), d["conv_pre"][j], rtol=0, atol=0.05)
        assert ok, f"layer {i} conv state after prefill differs by {err}"
    logits.clear()
    toks = d["tokens"]
    for step in range(5):
        eng.decode_step([0, 1], [int(toks[step][0]), int(toks[step][1])])   # teacher-forced
    h.remove()
    dec = torch.stack([lg for lg in logits]).numpy()
    err, ok = _close(dec, d["dec_logits"], rtol=0, atol=0.25)
    assert ok, f"decode logits differ by {err}"
    agree = (dec.argmax(-1) == d["dec_logits"].argmax(-1))
    margin = np.sort(d["dec_logits"], -1)[..., -1] - np.sort(d["dec_logits"], -1)[..., -2]
    assert agree[margin > 0.3].all()
    for j, i in enumerate(layers):
        err, ok = _close(eng.rec[i][:2].cpu(), d["rec_post"][j])
        assert ok, f"layer {i} recurrent state after decode differs by {err}"


def test_graph_decode_equals_eager_decode(setup):
    model, d = setup
    e1, e2 = _engine(model, graph=False), _engine(model, graph=True)
    for e in (e1, e2):
        e.prefill(1, torch.tensor(d["ids_a"], device=DEV)[None])
        e.prefill(0, torch.tensor(d["ids_b"], device=DEV)[None])
    t1 = t2 = [int(d["tokens"][0][0]), int(d["tokens"][0][1])]
    for _ in range(6):
        t1 = e1.decode_step([0, 1], t1)
        t2 = e2.decode_step([0, 1], t2)
        assert t1 == t2
    for i in e1.rec:
        assert torch.equal(e1.rec[i], e2.rec[i]) and torch.equal(e1.conv[i], e2.conv[i])


def test_packed_batch_prefill_equals_single_prefills(setup):
    model, d = setup
    e1, e2 = _engine(model), _engine(model)
    a = torch.tensor(d["ids_a"], device=DEV)[None]
    b = torch.tensor(d["ids_b"], device=DEV)[None]
    f1 = [e1.prefill(1, a), e1.prefill(0, b)]
    f2 = e2.prefill_batch([1, 0], [a, b])
    assert f1 == f2
    for i in e1.rec:
        assert _close(e1.rec[i][:2].cpu(), e2.rec[i][:2].cpu())[1]
        assert _close(e1.conv[i][:2].float().cpu(), e2.conv[i][:2].float().cpu(), rtol=0, atol=0.05)[1]
    assert e1.lens == e2.lens


def test_chunked_prefill_equals_whole_prefill(setup):
    """Chunked prefill (src/cb_tp.py:195-271) with state carried through the slot == one prefill;
    the other slot keeps decoding between chunks and its state is not disturbed (no hold needed)."""
    model, d = setup
    a = torch.tensor(d["ids_a"], device=DEV)[None]
    b = torch.tensor(d["ids_b"], device=DEV)[None]
    ref = _engine(model)
    ref.prefill(1, a)
    for c in (5, 16, 37):
        e = _engine(model)
        tb = [e.prefill(0, b)]
        first = None
        for p in range(0, a.shape[1], c):
            last = p + c >= a.shape[1]
            f = e.prefill_chunk(1, a[:, p:p + c], p, last)
            if last:
                first = f
            else:
                before = {i: e.rec[i][1].clone() for i in e.rec}
                tb.append(e.decode_step([0], [tb[-1]], hold=(1,))[0])
                for i in e.rec:
                    assert torch.equal(before[i], e.rec[i][1])
        assert first is not None
        for i in ref.rec:
            err, ok = _close(e.rec[i][1].cpu(), ref.rec[i][1].cpu())
            assert ok, f"chunk {c}: layer {i} state differs by {err}"
            assert _close(e.conv[i][1].float().cpu(), ref.conv[i][1].float().cpu(), rtol=0, atol=0.05)[1]
        assert e.lens[1] == ref.lens[1]


def test_patch_model_hf_forward_matches_unpatched(setup):
    """patch_model (src/cb_engine.py:54-77) installs the CUDA operators on HF's modules: HF's own
    forward, prefill then cached decode, gives the same logits as the unpatched torch fallbacks."""
    from transformers import DynamicCache
    model, d = setup
    patch = pkg("patch")
    ids = torch.tensor(d["ids_a"], device=DEV)[None]

    def run(m):
        cache = DynamicCache(config=m.config.text_config)
        with torch.inference_mode():
            out = m(input_ids=ids, past_key_values=cache, use_cache=True)
            lg = [out.logits[0, -1].float()]
            nxt = out.logits[0, -1].argmax()[None, None]
            for _ in range(3):
                out = m(input_ids=nxt, past_key_values=cache, use_cache=True)
                lg.append(out.logits[0, -1].float())
                nxt = out.logits[0, -1].argmax()[None, None]
        return torch.stack(lg)

    ref = run(model)
    import copy
    m2 = copy.deepcopy(model)
    assert patch.patch_model(m2, fast_gdn=True, gdn_v2=True) == 3
    got = run(m2)
    assert (got - ref).abs().max().item() < 0.25


def test_engine_raises_on_device_error_flag(setup):
    """A slot index outside the pools reaches the GDN kernels (decode and prefill): they record
    error 1 in the engine's device flag and leave every pool row as it was, and the engine raises
    RuntimeError at the step's own host read instead of returning silent garbage."""
    model, _ = setup
    eng = _engine(model)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, model.config.text_config.vocab_size, (1, 9), generator=g)
    eng.prefill(0, ids)
    eng.check_errors()                                   # a clean step leaves the flag at 0
    pools = [t.clone() for t in eng.rec.values()] + [t.clone() for t in eng.conv.values()]
    eng._pos.zero_()
    eng._slot.fill_(eng.N + 5)                           # past the scratch row: out of range
    with torch.inference_mode():
        out = eng._core(8)
    torch.cuda.synchronize()
    assert int(out[-1]) == 1                             # the flag rides with the step's tokens
    after = [t for t in eng.rec.values()] + [t for t in eng.conv.values()]
    assert all(torch.equal(a, b) for a, b in zip(pools, after))
    with pytest.raises(RuntimeError, match="slot index"):
        eng.check_errors()
    eng.check_errors()                                   # raising clears the flag
    # the same through the public prefill call: the GDN layers come first in this model, their
    # kernels flag the slot before any host-side indexing of the attention cache
    assert model.config.text_config.layer_types[0] == "linear_attention"
    with pytest.raises((RuntimeError, IndexError)):
        eng.prefill_batch([eng.N + 3], [ids])
    eng._err.zero_()
    assert eng.decode_step([0], [3])                     # the engine still runs after the error
