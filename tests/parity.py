"""Parity checks shared by the GPU tests: the north-star bounds, calibrated where the
reference's own BF16 rounding exceeds them, with every measured figure recorded.

  logits   |diff| <= 2e-2 absolute, or 2x the step's BF16-vs-FP32 spread of the reference
  greedy   teacher-forced along the reference's ids: a differing argmax only at a near-tie
           (top-1 / top-2 margin of the reference within twice the step's bound);
           free-running: equal up to the first flip, which must be such a near-tie
  state    rel-L2 <= 1e-3, or 2x the reference's BF16-vs-FP32 spread of the written state
  update   W' - W rel-L2 <= 3e-2

Why 2x the spread: the kernels are a second BF16 implementation of the same FP32 math, with
their own accumulation order and fusion.  If each BF16 implementation sits within the spread
of the FP32 result, the two can sit up to twice the spread apart (on opposite sides of it),
so that is the distance at which ours is still as accurate as the reference's own BF16 path.
The absolute floors (2e-2, 1e-3) are the north-star bounds themselves.
"""

import numpy as np

from conftest import record
from oracle.numerics import rel_l2

LOGIT_TOL = 2e-2
STATE_TOL = 1e-3
SPREAD_FACTOR = 2.0
NAMES = ("w_up", "w_gate", "w_down")


def _mask(logits, limit):
    w = np.asarray(logits, np.float64).copy()
    w[:6] = -np.inf
    w[limit:] = -np.inf
    return w


def masked_margin(logits, limit):
    w = _mask(logits, limit)
    top = np.sort(w)[-2:]
    return float(top[1] - top[0]), int(np.argmax(w))


def check_logits(name, ours, ref, spread, ids, limit):
    """Teacher-forced logits along the reference's ``ids``: every step within its bound, every
    greedy flip at a near-tie.  Returns (steps compared, flips)."""
    errs, bounds, flips = [], [], []
    for step, (o, r) in enumerate(zip(ours, ref)):
        o = np.asarray(o, np.float64)
        bound = max(LOGIT_TOL, SPREAD_FACTOR * spread[step])
        err = float(np.max(np.abs(o - r)))
        errs.append(err)
        bounds.append(bound)
        assert err <= bound, (name, step, err, spread[step])
        if int(np.argmax(_mask(o, limit))) != ids[step]:
            margin, _ = masked_margin(r, limit)
            flips.append(step)
            assert margin <= 2 * bound, (name, step, margin)
    record(name, steps_compared=len(errs), max_abs_logit_diff=max(errs),
           steps_over_2e2=sum(e > LOGIT_TOL for e in errs), max_bound=max(bounds), flips=flips)
    return len(errs), flips


def check_free_running(name, got, ref_ids, ref_logits, spread, limit):
    """Free-running greedy ids equal the reference's up to the first flip, which must be a near-tie."""
    first = None
    for step, (a, b) in enumerate(zip(got, ref_ids)):
        if a != b:
            first = step
            margin, _ = masked_margin(ref_logits[step], limit)
            bound = max(LOGIT_TOL, SPREAD_FACTOR * spread[step])
            assert margin <= 2 * bound, (name, step, margin)
            break
    assert len(got) == len(ref_ids)
    record(name, free_running_equal_steps=len(ref_ids) if first is None else first)
    return first


def check_state(name, new, ref, base, spread, extra=None):
    """Written FP32 masters against the reference's (``ref``), and against its FP32 run
    (``extra``) when given; ``spread`` holds the reference's own BF16-vs-FP32 distance."""
    for n in NAMES:
        got = getattr(new, n).detach().float().cpu().numpy()
        bound = max(STATE_TOL, SPREAD_FACTOR * spread[n])
        r = rel_l2(got, ref[n])
        u = rel_l2(got - base[n], ref[n] - base[n])
        record(name, **{f"{n}_state": r, f"{n}_state_bound": bound, f"{n}_update": u,
                        f"{n}_bf16_fp32_spread": spread[n]})
        assert r <= bound, (name, n, r, bound)
        assert u <= 3e-2, (name, n, u)
        if extra is not None:
            r32 = rel_l2(got, extra[n])
            record(name, **{f"{n}_state_vs_fp32": r32})
            assert r32 <= bound, (name, n, "vs FP32", r32, bound)


