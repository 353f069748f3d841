"""Pins the CPU oracle (oracle/gdn_oracle.c) to the contest reference.

The fixtures in tests/golden/gdn_golden.npz are inputs and outputs of the
contest's pure-torch reference (flashinfer-python 0.6.11.post2,
flashinfer/trace/templates/gdn.py), written by tests/golden/make_golden.py.
The oracle computes in fp32 like the reference, in a different summation
order, so the state agrees to ~1e-6 and the bf16 output to within one bf16
rounding step.
"""
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from parity import bf16_from_u16

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gdn_golden.npz")


def _load():
    z = np.load(GOLD)
    cases = {}
    for key in z.files:
        name, field = key.split("/")
        cases.setdefault(name, {"__name__": name})[field] = z[key]
    return cases


CASES = _load()
BF16_FIELDS = {"q", "k", "v", "a", "b", "out"}
BF16_STATE_CASES = {"mtp_bf16state_t1", "mtp_bf16state_t3"}


def _t(case, field):
    if field not in case:
        return None
    arr = case[field]
    if field in BF16_FIELDS or (field in ("initial_state", "new_state") and _name(case) in BF16_STATE_CASES):
        return bf16_from_u16(arr)
    return torch.from_numpy(np.array(arr))


def _name(case):
    return case.get("__name__")


def _check(o, s, case):
    ref_o = _t(case, "out").float()
    ref_s = _t(case, "new_state")
    o = o.float()
    if ref_s.dtype == torch.bfloat16:
        # bf16 state: identical except where the fp32 value sits on a rounding boundary
        d = (s.float() - ref_s.float()).abs()
        assert s.dtype == torch.bfloat16
        assert float((d <= 1e-7 + 2 ** -7 * ref_s.float().abs()).float().mean()) == 1.0
        assert float((d == 0).float().mean()) >= 0.98
        s, ref_s = ref_s.float(), ref_s.float()
    # state: fp32 vs fp32 in another summation order
    err = (s - ref_s).abs()
    assert float(err.max()) <= 1e-5 * float(ref_s.abs().max()) + 1e-6, float(err.max())
    # output: bf16 -- identical except where the fp32 value sits on a rounding boundary
    d = (o - ref_o).abs()
    assert float((d <= 1e-6 + 2 ** -7 * ref_o.abs()).float().mean()) == 1.0
    assert float((d == 0).float().mean()) >= 0.98


def test_golden_file_present():
    assert len([c for c in CASES if c.startswith("dec_")]) >= 4
    assert len([c for c in CASES if c.startswith("pre_")]) >= 4
    assert len([c for c in CASES if c.startswith("mtp_")]) >= 4
    assert len([c for c in CASES if c.startswith("ckpt_")]) >= 2
    assert len([c for c in CASES if c.startswith("pre_l2norm")]) >= 2


@pytest.mark.parametrize("name", sorted(c for c in CASES if c.startswith("dec_")))
def test_oracle_decode_matches_reference(name):
    c = CASES[name]
    args = [_t(c, f) for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")]
    o, s = oracle.decode(*args, float(c["scale"]))
    _check(o, s, c)


@pytest.mark.parametrize("name", sorted(c for c in CASES if c.startswith("pre_")))
def test_oracle_prefill_matches_reference(name):
    c = CASES[name]
    args = [_t(c, f) for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")]
    l2 = bool(int(c["qk_l2norm"])) if "qk_l2norm" in c else False
    o, s = oracle.prefill(*args, float(c["scale"]), qk_l2norm=l2)
    _check(o, s, c)


def test_oracle_prefill_l2norm_is_not_a_no_op():
    """The l2norm cases feed raw q/k: without the flag the oracle misses."""
    c = CASES["pre_l2norm"]
    args = [_t(c, f) for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")]
    o, s = oracle.prefill(*args, float(c["scale"]), qk_l2norm=False)
    # (raw vectors of norm ~17 make the recurrence diverge; NaN compares unequal)
    assert not torch.allclose(s, _t(c, "new_state"), rtol=1e-2, atol=1e-2)


MTP_FIELDS = ("q", "k", "v", "initial_state", "initial_state_indices", "A_log", "a", "dt_bias", "b")


def _mtp_args(c):
    return [_t(c, f) for f in MTP_FIELDS]


@pytest.mark.parametrize("name", sorted(c for c in CASES if c.startswith("mtp_")))
def test_oracle_mtp_matches_reference(name):
    c = CASES[name]
    buf = torch.zeros_like(_t(c, "intermediate")) if "intermediate" in c else None
    o, s = oracle.mtp(*_mtp_args(c), float(c["scale"]), buf, qk_l2norm=bool(c["qk_l2norm"]))
    _check(o, s, c)
    if buf is not None:
        ref = _t(c, "intermediate")
        assert float((buf - ref).abs().max()) <= 1e-5 * float(ref.abs().max()) + 1e-6
    # slots no batch entry names are passed through unchanged
    used = set(int(i) for i in c["initial_state_indices"])
    for slot in range(s.shape[0]):
        if slot not in used:
            assert torch.equal(s[slot], _t(c, "initial_state")[slot])


def test_oracle_mtp_padding_rule():
    """An index outside [0, pool) is padding: zero output, no state touched;
    the other entries are unaffected by it."""
    c = CASES["mtp_small"]
    args = _mtp_args(c)
    idx = args[4].clone()
    idx_pad = idx.clone()
    idx_pad[1] = -1
    o_ref, s_ref = oracle.mtp(*args[:4], idx, *args[5:], float(c["scale"]))
    o, s = oracle.mtp(*args[:4], idx_pad, *args[5:], float(c["scale"]))
    assert not o[1].float().any()
    assert torch.equal(o[0], o_ref[0]) and torch.equal(o[2], o_ref[2])
    pool = args[3]
    assert torch.equal(s[int(idx[1])], pool[int(idx[1])])
    assert torch.equal(s[int(idx[0])], s_ref[int(idx[0])])
    idx_pad[1] = pool.shape[0]  # one past the end is padding too
    o2, s2 = oracle.mtp(*args[:4], idx_pad, *args[5:], float(c["scale"]))
    assert torch.equal(o2, o) and torch.equal(s2, s)


@pytest.mark.parametrize("name", sorted(c for c in CASES if c.startswith("ckpt_")))
def test_oracle_prefill_checkpoints_match_reference(name):
    c = CASES[name]
    args = [_t(c, f) for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")]
    every = int(c["every"])
    o, s, ck = oracle.prefill(*args, float(c["scale"]), checkpoint_every_n_tokens=every)
    _check(o, s, c)
    assert torch.equal(oracle.checkpoint_cu_starts(args[8], every),
                       torch.from_numpy(c["checkpoint_cu_starts"]))
    ref = _t(c, "checkpoints")
    assert ck.shape == ref.shape
    assert float((ck - ref).abs().max()) <= 1e-5 * float(ref.abs().max()) + 1e-6


def test_golden_covers_edge_cases():
    # a zero-length sequence keeps a zero state even with an initial state given
    c = CASES["pre_varlen_empty"]
    cu = c["cu_seqlens"]
    empty = [i for i in range(len(cu) - 1) if cu[i + 1] == cu[i]]
    assert empty and "state" in c
    for i in empty:
        assert not c["new_state"][i].any()
    # the softplus threshold and saturated sigmoid are exercised
    a = bf16_from_u16(CASES["dec_gva4_extreme"]["a"]).float()
    assert float(a.max()) > 20 and float(a.min()) < -20


def test_oracle_plants_are_caught():
    """A wrong gate or a wrong GVA mapping in the oracle must fail the golden check."""
    c = CASES["dec_small"]
    args = [_t(c, f) for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")]
    bad = list(args)
    bad[4] = args[4] + 0.5  # A_log off by 0.5
    o, s = oracle.decode(*bad, float(c["scale"]))
    with pytest.raises(AssertionError):
        _check(o, s, c)
    bad = list(args)
    bad[0] = args[0].flip(2)  # q heads swapped
    bad[1] = args[1].flip(2)
    o, s = oracle.decode(*bad, float(c["scale"]))
    with pytest.raises(AssertionError):
        _check(o, s, c)


def test_oracle_mtp_snapshots_by_entry_are_a_reindexing():
    """Snapshots by batch entry (flashinfer's kernel, row i * T + t) hold the
    same states as the golden-pinned by-slot snapshots (the contest
    definition), moved from slot idx[i] to entry i; padding entries and
    entries whose rows do not fit write nothing."""
    B, T, pool, H, HV, K = 4, 3, 6, 1, 2, 16
    g = torch.Generator().manual_seed(7)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, K, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, HV, K, generator=g).to(torch.bfloat16)
    st = torch.randn(pool, HV, K, K, generator=g) * 0.1
    A_log = torch.rand(HV, generator=g)
    a = torch.randn(B, T, HV, generator=g).to(torch.bfloat16)
    dt = torch.rand(HV, generator=g) - 0.5
    b = torch.randn(B, T, HV, generator=g).to(torch.bfloat16)
    idx = torch.tensor([4, -1, 0, 5])
    by_slot = torch.zeros(pool, T, HV, K, K)
    oracle.mtp(q, k, v, st, idx, A_log, a, dt, b, 0.0, intermediate_states_buffer=by_slot)
    by_entry = torch.full((B, T, HV, K, K), 7.0)
    oracle.mtp(q, k, v, st, idx, A_log, a, dt, b, 0.0, intermediate_states_buffer=by_entry,
               snapshots_by_entry=True)
    for i, s in enumerate(idx.tolist()):
        if s < 0:
            assert torch.all(by_entry[i] == 7.0)
        else:
            assert torch.equal(by_entry[i], by_slot[s])
    # a buffer of 3 entries' rows with cache_steps = T + 1: rows i * T + t, entry 3 does not fit
    packed = torch.full((3, T + 1, HV, K, K), 7.0)
    oracle.mtp(q, k, v, st, idx, A_log, a, dt, b, 0.0, intermediate_states_buffer=packed,
               snapshots_by_entry=True)
    rows = packed.view(-1, HV, K, K)
    for i, s in enumerate(idx.tolist()):
        for t in range(T):
            r = i * T + t
            if s >= 0 and (i + 1) * T <= rows.shape[0]:
                assert torch.equal(rows[r], by_slot[s, t])
            elif r < rows.shape[0]:
                assert torch.all(rows[r] == 7.0)
