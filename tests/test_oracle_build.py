"""CPU: the oracle's index build (initialize / grouping levels / assemble,
DS/runtime.py:170-233) against the reference's own kernels run in the Triton
interpreter (tests/golden/build.npz), and the grouping ops against the
known-answer cases of NA/test_fused_grouping_small.py restated here."""
import numpy as np

from oracle import v1x_oracle as O


def _interpreter_cast_defect(mine, ref):
    """The two ways the Triton interpreter's float8e4nv cast departs from
    round-to-nearest-even (the hardware conversion and torch's cast, which the
    oracle follows), both rounding the magnitude down where RTNE rounds up:
    (a) the carry from the mantissa into the exponent is lost (31.7 -> 16
    instead of 32): same sign, `mine` a power-of-two code (mantissa bits 0),
    `ref` one exponent step (8 codes) lower; (b) subnormals are truncated
    toward zero (1.74 ulp -> 1 instead of 2): both subnormal, same sign, `ref`
    one code lower."""
    mine = mine.astype(np.int32)
    ref = ref.astype(np.int32)
    same_sign = (mine & 0x80) == (ref & 0x80)
    carry = ((mine & 7) == 0) & ((mine & 0x7F) - (ref & 0x7F) == 8)
    subnormal = ((mine & 0x78) == 0) & ((ref & 0x78) == 0) & ((mine & 7) - (ref & 7) == 1)
    return same_sign & (carry | subnormal)


def test_build_bucket_golden(golden):
    g = golden("build")
    for b in range(2):
        unit, perm0 = O.build_initialize(g["native"], g["tables"][b])
        assert np.array_equal(unit.view(np.uint32), g[f"unit{b}"].view(np.uint32))
        assert np.array_equal(perm0, np.arange(1024))
        perm = O.group_bucket(unit)
        assert np.array_equal(perm, g[f"perm{b}"])
        tmp, centers, mapping = O.build_assemble(g["native"], g["tables"][b], int(g["starts"][b]), perm)
        assert np.array_equal(tmp, g[f"tmp{b}"])
        assert np.array_equal(mapping, g[f"mapping{b}"])
        # scales exact; bytes exact except where the interpreter's cast is not RTNE
        assert np.array_equal(centers[:, 8192:], g[f"centers{b}"][:, 8192:])
        mine, ref = centers[:, :8192], g[f"centers{b}"][:, :8192]
        diff = mine != ref
        assert _interpreter_cast_defect(mine[diff], ref[diff]).all()
        assert diff.mean() < 0.05


def test_build_adversarial_ties(golden):
    """Bucket 1 holds duplicated tokens, zero tokens and a constant page: the
    grouping's argmin ties (leftmost) and sort ties (lower position) decide."""
    g = golden("build")
    unit, _ = O.build_initialize(g["native"], g["tables"][1])
    zero_rows = (unit == 0).all(1)
    assert zero_rows.sum() >= 20 and len(np.unique(unit, axis=0)) < 1000
    perm = O.group_bucket(unit)
    assert np.array_equal(perm, g["perm1"])
    assert sorted(perm.tolist()) == list(range(1024))


def test_e4m3_encoder_round_trip():
    codes = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_to_f32(codes)
    finite = ~np.isnan(vals)
    assert np.array_equal(O.e4m3_from_f32(vals[finite]), codes[finite])
    # halfway cases go to the even code; saturation at 448
    assert O.e4m3_from_f32(np.float32(17.0)) == O.e4m3_from_f32(np.float32(16.0))
    assert O.e4m3_from_f32(np.float32(19.0)) == O.e4m3_from_f32(np.float32(20.0))
    assert O.E4M3[O.e4m3_from_f32(np.float32(1000.0))] == 448.0
    assert O.e4m3_from_f32(np.float32(-0.0)) == 0x80


def test_e4m3_encoder_matches_torch_cast():
    import torch
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 1e-2, 1.0, 30.0, 200.0)]).astype(np.float32)
    x = np.clip(x, -448, 448)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_from_f32(x), want)


def test_pow2_ceil():
    v = np.array([1.0, 1.5, 0.25, 3.0e-7, 0.7, 2.0 ** -20 * 1.0000001], np.float32)
    got = O.pow2_ceil(v)
    exp = np.array([1.0, 2.0, 0.25, 2.0 ** -21, 1.0, 2.0 ** -19], np.float32)
    assert np.array_equal(got, exp)


# -- known answers of the reference's grouping tests (NA/test_fused_grouping_small.py) --

def test_dots_three_modes():
    """Member ids, not positions, select the vectors; MODE 2 subtracts S."""
    start = 100
    unit = np.zeros((16, 128), np.float32)
    signs = np.array([1, -1] * 8, np.float32)
    unit[:, 0] = signs
    order = [2, 1, 4, 3, 6, 5, 8, 7, 10, 9, 12, 11, 14, 13, 0, 15]
    P = np.array([start + i for i in order], np.int32)
    A = np.zeros(512, np.int32)
    A[0:2] = [start + 1, start + 2]   # b negative, a positive
    for mode in (0, 1, 2):
        S = -signs[order] if mode == 2 else np.zeros(16, np.float32)
        out = O.group_dots(unit, P, A, S, 16, start, mode, count=16)
        exp = [(1 if i % 2 == 0 else -1) * [1, -1, 2][mode] for i in order]
        assert np.array_equal(out, np.array(exp, np.float32))


def test_anchor_left_tie():
    P = np.array([115, 101, 102, 100] + list(range(103, 115)), np.int32)
    S = np.array([4, -3, 2, -3] + [5] * 12, np.float32)
    A = np.full(512, -99, np.int32)
    for slot in (0, 1):
        A = O.group_anchor(P, A, S, 16, slot, count=16)
    assert A[:2].tolist() == [101, 101]   # leftmost minimum (position 1), not the smaller id


def test_one_split_chain():
    unit = np.zeros((16, 128), np.float32)
    unit[:, 0] = [1, -1] * 8
    P = np.arange(100, 116, dtype=np.int32)
    A = np.zeros(512, np.int32)
    S = np.zeros(16, np.float32)
    for mode in (0, 1, 2):
        S = O.group_dots(unit, P, A, S, 16, 100, mode, count=16)
        if mode < 2:
            A = O.group_anchor(P, A, S, 16, mode, count=16)
    out = O.sort_segments(P, S, -1, 16, 1, 1, O=np.zeros_like(P))
    assert A[:2].tolist() == [101, 100]
    assert out.tolist() == list(range(100, 116, 2)) + list(range(101, 116, 2))
