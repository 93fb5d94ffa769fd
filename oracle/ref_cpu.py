"""The reference's own GDN functions, imported from ``oracle/_ref`` for the timed CPU baselines.

Test and baseline infrastructure: ``oracle/install_ref.py`` installs the reference's modules into
``oracle/_ref`` (git-ignored; it travels with working-tree snapshots).  When they are there, this
module imports them, with the two stand-ins the reference needs off Ascend hardware (an empty
``torch_npu`` module registered after transformers loads, and transformers told that no NPU is
present), and exposes:

  * ``chunk_prefill(q, k, v, g, beta, init)`` -- fast_chunk_gated_delta_rule_v2
    (src/gdn_chunk_fast2.py:11-62) for one sequence, q/k already repeated to the value heads;
  * ``decode_layer(...)`` -- the operator sequence of CBEngine._gdn (src/cb_engine.py:318-352) for
    the slots of one layer: elem_conv_update (src/cb_engine.py:43-51), split, beta / g, GQA repeat,
    recurrent_single_step (src/recurrent_single_step.py:8-32) on the dense pool, and HF's
    Qwen3_5RMSNormGated (the oracle of the reference's closed npu norm).

``available()`` is False when ``oracle/_ref`` does not hold the reference; bench.py then times the
torch restatement in ``gdn_torch_cpu.py`` instead and says so (``kind: "port"``).
"""
from __future__ import annotations

import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_mods = None


def _load():
    global _mods
    if _mods is not None:
        return _mods or None
    if not os.path.exists(os.path.join(REF_DIR, "gdn_chunk_fast2.py")):
        _mods = {}
        return None
    import transformers.utils.import_utils as iu
    iu.is_torch_npu_available = lambda *a, **k: False
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M  # (imported before the stand-in)
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import cb_engine
    import gdn_chunk_fast2
    import recurrent_single_step
    _mods = dict(M=M, v2=gdn_chunk_fast2.fast_chunk_gated_delta_rule_v2,
                 rec=recurrent_single_step.recurrent_single_step, elem=cb_engine.elem_conv_update)
    return _mods


def available() -> bool:
    return _load() is not None


def chunk_prefill(q, k, v, g, beta, init):
    """One sequence through the reference's v2 chunk rule: q, k, v [1, L, H, d] (bf16), g fp32 and
    beta (bf16) [1, L, H], init [1, H, dk, dv] fp32.  Returns (out, final state)."""
    m = _load()
    return m["v2"](q, k, v, g, beta, 64, init, True, True)


class _Norm:
    """HF's Qwen3_5RMSNormGated with the given weight (built once per weight)."""

    def __init__(self, M, w, eps):
        import torch
        self.mod = M.Qwen3_5RMSNormGated(w.shape[0], eps=eps)
        with torch.no_grad():
            self.mod.weight.copy_(w.float())
        self.mod = self.mod.to(w.dtype)

    def __call__(self, x, z):
        return self.mod(x, z)


def decode_layer(mixed, z, a, b, A_log, dt_bias, conv_w, conv_pool, rec_pool, norm_w, Hk, Hv, d, eps=1e-6):
    """CBEngine._gdn's operators (src/cb_engine.py:318-352) for the n slots of the pools, in pool
    order as the reference's dense decode runs them; conv_pool and rec_pool are updated in place."""
    import torch
    import torch.nn.functional as F
    m = _load()
    n = mixed.shape[0]
    y = m["elem"](mixed[:, :, None], conv_pool, conv_w, None)[:, :, 0]
    q = y[:, :Hk * d].reshape(n, 1, Hk, d)
    k = y[:, Hk * d:2 * Hk * d].reshape(n, 1, Hk, d)
    v = y[:, 2 * Hk * d:].reshape(n, 1, Hv, d)
    beta = b.sigmoid()[:, None]
    g = (-A_log.float().exp() * F.softplus(a.float() + dt_bias))[:, None]
    r = Hv // Hk
    q, k = q.repeat_interleave(r, dim=2), k.repeat_interleave(r, dim=2)
    core, S = m["rec"](q, k, v, g=g, beta=beta, initial_state=rec_pool, output_final_state=True,
                       use_qk_l2norm_in_kernel=True)
    rec_pool.copy_(S.to(rec_pool.dtype))
    norm = _Norm(m["M"], norm_w, eps)
    return norm(core.reshape(-1, d), z.reshape(-1, d)).reshape(n, Hv, d)
