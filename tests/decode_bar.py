"""The decode block's parity bar, shared by the GPU tests of the fused decode kernels.

moe_combine (strata_mlx/fused.py:467-481) rounds two terms to the activations' type and adds them: the routed sum
OutT(sum_k y_k w_k) and the gated shared output OutT(OutT(sigmoid(g)) s). A float32 sum on the GPU and the oracle's
float64 sum may round a product y_k (or a term) one unit of the type apart, so the bar is stated in units of the
terms the combine adds: |got - want| <= 2 units of M + 1 unit of |want|, M the largest of |routed|, |shared| and
w_k |y_k|; the last unit is the final rounding of the sum.

One exception, checked: where the shared gate OutT(sigmoid(g)) sits on a rounding edge of the type (its logit or
its sigmoid one unit away gives another rounded gate), CUDA's expf and numpy's exp may round it apart. Such an
element passes if it meets the bar against the oracle recomputed with the neighbouring gate.
"""

import numpy as np

from oracle import blocks_ref as R

MANT = {"bfloat16": 7, "float16": 10}


def unit(v: np.ndarray, dt: str) -> np.ndarray:
    """One unit in the last place of the type at |v| (the smallest normal's unit for values below it)."""
    m = MANT[dt]
    lo = -126 if dt == "bfloat16" else -14
    e = np.floor(np.log2(np.maximum(np.abs(v), 2.0 ** lo)))
    return 2.0 ** (e - m)


def bar(parts: dict, dt: str) -> np.ndarray:
    yk = np.abs(parts["y"]) * parts["w"][..., None]
    M = np.maximum(np.maximum(np.abs(parts["routed"]), np.abs(parts["shared"])), yk.max(axis=-2))
    return 2 * unit(M, dt) + unit(parts["out"], dt)


def neighbour_gates(gs: np.ndarray, dt: str) -> list:
    """Gates one step off the oracle's: the logit a unit of the type either way, and the float32 sigmoid one
    float32 ulp either way, each rounded to the type; only values that differ from the oracle's gate."""
    g0 = R.gate_of(gs.reshape(-1, 1), dt)
    out = []
    u = unit(gs, dt).reshape(-1, 1).astype(np.float32)
    for g in (gs.reshape(-1, 1) - u, gs.reshape(-1, 1) + u):
        out.append(R.gate_of(g, dt))
    with np.errstate(over="ignore"):
        sig = (np.float32(1) / (np.float32(1) + np.exp(-gs.reshape(-1, 1).astype(np.float32)))).astype(np.float32)
    for d in (-np.inf, np.inf):
        out.append(R.round_to(np.nextafter(sig, np.float32(d)).astype(np.float32), dt))
    return [g for g in out if not np.array_equal(g, g0)]


def check(got: np.ndarray, parts: dict, dt: str) -> dict:
    """Asserts the bar for every output; returns counts (elements checked, elements that took the gate exception)."""
    want = parts["out"]
    tol = bar(parts, dt)
    ok = np.abs(got - want) <= tol
    excused = np.zeros_like(ok)
    if not ok.all():
        for g in neighbour_gates(parts["gs"], dt):
            alt = R.moe_combine_parts(parts["y"], parts["w"], parts["gs"], parts["s"], dt, gate=g)
            alt["y"], alt["w"] = parts["y"], parts["w"]
            fine = (~ok) & (np.abs(got - alt["out"]) <= bar(alt, dt))
            # the exception is only for tokens whose gate this neighbour changes
            changed = (g != parts["gate"]).reshape(-1, 1)
            excused |= fine & changed
    bad = ~(ok | excused)
    if bad.any():
        t, c = np.nonzero(bad)
        i = np.argmax(np.abs(got - want)[bad] / tol[bad])
        raise AssertionError(
            f"{bad.sum()} of {bad.size} outputs beyond the bar; worst at token {t[i]}, row {c[i]}: got {got[t[i], c[i]]}, "
            f"oracle {want[t[i], c[i]]}, bar {tol[t[i], c[i]]:.3g} (routed {parts['routed'][t[i], c[i]]}, shared "
            f"{parts['shared'][t[i], c[i]]})")
    return {"checked": int(ok.size), "gate_exceptions": int(excused.sum())}
