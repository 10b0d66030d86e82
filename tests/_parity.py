"""Parity checks shared by the GPU tests (test infrastructure).

Outputs: bf16 values agree when |a - b| <= 2e-2 + 2e-2 |b| (the bf16 tolerance of
the parity target), and every element must agree: a failure names how many
elements are out, the largest error and where it is.

Routing: selections are integers and must be equal.  The one accepted exception
is a near-tie in the reference's own scores.  A score is a bf16 rounding of an
fp32 sum; summed in another order it can land one bf16 ulp away, so two scores
within two ulps of each other (each may move by one, in opposite directions) can
change places.  ``training_route_flips`` lists every query whose
selection differs, proves each difference is such a near-tie against the
oracle's scores, and the output check then exempts only those queries.
"""
import math

import torch

ATOL = RTOL = 2e-2


def out_of_tolerance(a, b, atol=ATOL, rtol=RTOL):
    a, b = a.float().cpu(), b.float().cpu()
    return (a - b).abs() > atol + rtol * b.abs()


def assert_close(a, b, what="output", exempt=None, atol=ATOL, rtol=RTOL):
    """Every element within tolerance, except those under ``exempt`` (a bool mask
    broadcastable to the shape: queries whose routing flipped at a near-tie)."""
    a, b = a.float().cpu(), b.float().cpu()
    assert a.shape == b.shape, (what, a.shape, b.shape)
    bad = out_of_tolerance(a, b, atol, rtol)
    if exempt is not None:
        bad &= ~exempt.expand_as(bad)
    n = int(bad.sum())
    if n:
        err = ((a - b).abs() - rtol * b.abs()).masked_fill(~bad, -1)
        idx = tuple(int(i) for i in torch.nonzero(err == err.max())[0])
        raise AssertionError(f"{what}: {n} of {a.numel()} elements out of tolerance; worst at {idx}: "
                             f"{a[idx].item()} vs {b[idx].item()}")


def bf16_ulp(x):
    """Spacing of bf16 values at |x| (8 significant bits)."""
    x = abs(float(x))
    if x == 0 or not math.isfinite(x):
        return 2.0 ** -133
    return 2.0 ** (math.floor(math.log2(x)) - 7)


def _near(a, b):
    """Within two bf16 ulps: each of two independently rounded scores may move one."""
    return abs(a - b) <= 2 * max(bf16_ulp(a), bf16_ulp(b))


def training_route_flips(gpu_sel, tiles, heads):
    """Compare the library's training selections with the oracle's.

    gpu_sel: int16 [B, T, H_all, mmax] (-1 padded) from the training forward;
    tiles: ``oracle.tao_oracle.training_routes`` on the inputs of ``heads``.
    Returns (flipped [B, T, len(heads), 1] bool, n_flipped, problems): problems
    lists every differing query whose difference is not a near-tie (must be empty).
    """
    b, t = gpu_sel.shape[:2]
    flipped = torch.zeros(b, t, len(heads), 1, dtype=torch.bool)
    problems = []
    sel_all = gpu_sel[:, :, heads].long().cpu()
    for info in tiles:
        r0, m = info["tile"] * 256, info["count"]
        ora = info["sel"]
        mine = sel_all[:, r0:r0 + ora.shape[1], :, :m]
        if torch.equal(mine, ora) and bool((sel_all[:, r0:r0 + ora.shape[1], :, m:] < 0).all()):
            continue
        diff = (mine != ora).any(-1)
        for bi, qi, hi in torch.nonzero(diff).tolist():
            flipped[bi, r0 + qi, hi] = True
            g, r = mine[bi, qi, hi].tolist(), ora[bi, qi, hi].tolist()
            score = info["fine_score"][bi, qi, hi]
            why = _explain(g, r, score, info, bi, qi, hi)
            if why:
                problems.append((bi, r0 + qi, heads[hi], why))
    return flipped, int(flipped.sum()), problems


def _explain(g, r, score, info, bi, qi, hi):
    """'' when the two selections differ only at near-ties of the oracle's scores."""
    if -1 in g:
        return f"library selected fewer than {len(r)} fines: {g}"
    thr = min(score[i].item() for i in r)
    page_thr = None
    if "chosen" in info:
        masses = info["page_mass"][bi, qi, hi]
        chosen = info["chosen"][bi, qi, hi].tolist()
        page_thr = min(masses[p].item() for p in chosen)
    def page_near_tie(fine):
        page = fine // 8
        if page >= info["completed"] or page_thr is None:
            return False
        return _near(info["page_mass"][bi, qi, hi][page].item(), page_thr)
    if set(g) == set(r):   # same fines, another order: neighbours must tie
        for a, c in zip(g, r):
            if a != c and not _near(score[a].item(), score[c].item()):
                return (f"order differs beyond a tie: {g} vs {r} (oracle scores of fines {a}, {c}: "
                        f"{score[a].item()}, {score[c].item()})")
        return ""
    for f in set(g) - set(r):
        if not (_near(score[f].item(), thr) or page_near_tie(f)):
            return f"fine {f} (score {score[f].item()}) chosen over threshold {thr}"
    for f in set(r) - set(g):
        if not (_near(score[f].item(), thr) or page_near_tie(f)):
            return f"fine {f} (score {score[f].item()}) dropped against threshold {thr}"
    return ""
