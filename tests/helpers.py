"""Problem builders shared by the GPU tests: seeded inputs quantised on the
host by the oracle (the checker), uploaded to the device for the kernels."""
import numpy as np
import torch


def mxfp8_problem(orc, m, n, k, seed, sf_mode="data", batch=1):
    """Returns host (qa, qb, sa, sb) lists per batch and device tensors."""
    qa_l, qb_l, sa_l, sb_l = [], [], [], []
    for b in range(batch):
        x = orc.normal((m, k), seed=seed * 1000 + 2 * b)
        w = orc.normal((n, k), seed=seed * 1000 + 2 * b + 1)
        qa, sa = orc.quant_mxfp8(x)
        qb, sb = orc.quant_mxfp8(w)
        sa, sb = scale_mode(sa, sf_mode), scale_mode(sb, sf_mode)
        qa_l.append(qa), qb_l.append(qb), sa_l.append(sa), sb_l.append(sb)
    return qa_l, qb_l, sa_l, sb_l


def mxfp4_problem(orc, m, n, k, seed, sf_mode="data"):
    x = orc.normal((m, k), seed=seed * 1000)
    w = orc.normal((n, k), seed=seed * 1000 + 1)
    qa, sa = orc.quant_mxfp4(x)
    qb, sb = orc.quant_mxfp4(w)
    return qa, qb, scale_mode(sa, sf_mode), scale_mode(sb, sf_mode)


def scale_mode(sf, mode):
    """The reference's fixture patterns: data-derived scales, all-127 (unit,
    MXFP8_UNIT_SCALE / MXFP4_UNIT_SCALE) or 120 + g % 13 (MXFP4_SFA_K_PATTERN)."""
    if mode == "data":
        return sf
    if mode == "unit":
        return np.full_like(sf, 127)
    if mode == "kpattern":
        g = np.arange(sf.shape[1])
        return np.tile((120 + g % 13).astype(np.uint8), (sf.shape[0], 1))
    if mode == "rowpattern":
        r = np.arange(sf.shape[0])[:, None]
        g = np.arange(sf.shape[1])[None, :]
        return (122 + (r * 3 + g * 5) % 11).astype(np.uint8)
    raise ValueError(mode)


def dev_u8(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def to_f32(out):
    return out.float().cpu().numpy()


# (what, elements passing only through the fp32-accumulation floor, elements,
#  max relative error, calc_diff) of every assert_close call in this session;
# conftest.py prints it at the end of the run
PARITY_LOG = []


def floor_only_count(ref, got, mag):
    """Elements within 2^-7|ref| + 1e-3 + 1e-6*sum|term| but NOT within the
    target rule 2^-7|ref| + 1e-3 alone: the ones the floor lets through."""
    if mag is None:
        return 0
    err = np.abs(np.asarray(got, np.float64) - ref)
    base = (2.0 ** -7) * np.abs(ref) + 1e-3
    return int(np.count_nonzero((err > base) & (err <= base + 1e-6 * mag)))


def assert_close(orc, ref, got, mag=None, what=""):
    """Tolerance of every parity test (bf16 outputs):
         |err| <= 2^-7 |ref| + 1e-3 + 1e-6 * sum|a*b*s|   per element,
         max relative error <= 1e-2 over non-cancelling elements.
    The target rule plus an fp32-accumulation floor; see
    oracle.check_baseline_rule.  The number of elements that pass only
    through the floor is logged in PARITY_LOG."""
    bad, max_rel, calc_diff = orc.check_baseline_rule(ref, got, mag)
    PARITY_LOG.append((what, floor_only_count(ref, got, mag), int(np.size(ref)), max_rel, calc_diff))
    if bad:
        err = np.abs(got.astype(np.float64) - ref)
        floor = 0.0 if mag is None else 1e-6 * mag
        idx = np.unravel_index(np.argmax(err - (2.0 ** -7) * np.abs(ref) - floor), ref.shape)
        raise AssertionError(
            f"{what}: {bad} / {ref.size} elements out of tolerance; worst at {idx}: "
            f"ref={ref[idx]!r} got={got[idx]!r} mag={None if mag is None else mag[idx]!r}; "
            f"calc_diff={calc_diff:.3e}")
    assert max_rel <= 1e-2, f"{what}: max rel err {max_rel}"
    return calc_diff
