"""The oracle is the ground truth for the kernels, so it is pinned to the reference itself.

Golden vectors in tests/golden/ were produced by kernel-lab's own ``reference.py`` and
``kv_cache.py`` (tests/golden/make_golden.py). Here the NumPy oracle must reproduce them,
and this repository's fixture builder must reproduce the reference's inputs bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.conftest import (
    DT,
    build_decode_case,
    golden_array,
    golden_index,
    golden_to_torch,
    make_rms_inputs,
    sha,
    to_f32_numpy,
)

DECODE_CASES = [c["name"] for c in golden_index()["decode"]]
RMS_CASES = [c["name"] for c in golden_index()["rmsnorm"]]
ORACLE_TOL = {"f32": 1e-5, "f16": 1e-3, "bf16": 8e-3}


def _decode(name):
    return next(c for c in golden_index()["decode"] if c["name"] == name)


def _rms(name):
    return next(c for c in golden_index()["rmsnorm"] if c["name"] == name)


@pytest.mark.parametrize("name", DECODE_CASES)
def test_builder_reproduces_reference_inputs(name):
    case = _decode(name)
    q, kv, _, _ = build_decode_case(case, poison=1e4)
    got = {
        "q": sha(q),
        "k_cache": sha(kv.k_cache),
        "v_cache": sha(kv.v_cache),
        "block_table": sha(kv.block_table),
        "seq_lens": sha(kv.seq_lens),
    }
    assert got == case["in_sha256"]


@pytest.mark.parametrize("name", DECODE_CASES)
def test_oracle_decode_matches_reference(name):
    case = _decode(name)
    q, kv, _, _ = build_decode_case(case)  # NaN-poisoned spares: never read
    got = oracle.paged_decode_attention(
        to_f32_numpy(q), to_f32_numpy(kv.k_cache), to_f32_numpy(kv.v_cache), kv.block_table.numpy(),
        kv.seq_lens.numpy(), case.get("scale"), case["dt"],
    )
    want = golden_to_torch(golden_array("decode", f"{name}/out"), case["dt"]).float().numpy()
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, atol=ORACLE_TOL[case["dt"]], rtol=ORACLE_TOL[case["dt"]])


def test_oracle_known_answer_one_hot_key():
    """One key far more aligned than the rest and v[t] = t: the output is 13.0 (reference test
    tests/test_paged_attention.py:81-91)."""
    from kernel_lab.kv_cache import build_paged_kv

    d = 32
    keys = [torch.zeros(20, 1, d)]
    values = [torch.arange(20, dtype=torch.float32)[:, None, None].expand(20, 1, d).clone()]
    keys[0][13, 0, 0] = 100.0
    kv = build_paged_kv(keys, values, page_size=16, poison=1e4)
    assert {
        "k_cache": sha(kv.k_cache),
        "v_cache": sha(kv.v_cache),
        "block_table": sha(kv.block_table),
    } == golden_index()["onehot"]["in_sha256"]
    q = np.zeros((1, 1, d), np.float32)
    q[0, 0, 0] = 1.0
    out = oracle.paged_decode_attention(
        q, kv.k_cache.numpy(), kv.v_cache.numpy(), kv.block_table.numpy(), kv.seq_lens.numpy(), scale=1.0
    )
    np.testing.assert_allclose(out, golden_array("decode", "onehot/out"), atol=1e-5)
    np.testing.assert_allclose(out, 13.0, atol=1e-4)


@pytest.mark.parametrize("name", RMS_CASES)
def test_oracle_rmsnorm_matches_reference(name):
    case = _rms(name)
    dt = case["dt"]
    x, r, w = make_rms_inputs(case["shape"], DT[dt])
    assert {"x": sha(x), "residual": sha(r), "weight": sha(w)} == case["in_sha256"]
    out, new_res = oracle.fused_add_rms_norm(to_f32_numpy(x), to_f32_numpy(r), to_f32_numpy(w), case["eps"], dt)
    plain = oracle.rms_norm(to_f32_numpy(x), to_f32_numpy(w), case["eps"], dt)
    # Residual: bit-exact against the reference's hash.
    assert sha(torch.from_numpy(new_res).to(DT[dt])) == case["residual_out_sha256"]
    tol = {"f32": 1e-5, "f16": 2e-3, "bf16": 1.6e-2}[dt]
    if "sample_rows" in case:
        rows = case["sample_rows"]
        h = case["shape"][-1]
        want = golden_to_torch(golden_array("rmsnorm", f"{name}/out_rows"), dt).float().numpy()
        want_plain = golden_to_torch(golden_array("rmsnorm", f"{name}/out_plain_rows"), dt).float().numpy()
        np.testing.assert_allclose(out.reshape(-1, h)[rows], want, atol=tol, rtol=tol)
        np.testing.assert_allclose(plain.reshape(-1, h)[rows], want_plain, atol=tol, rtol=tol)
    else:
        want = golden_to_torch(golden_array("rmsnorm", f"{name}/out"), dt).float().numpy()
        want_plain = golden_to_torch(golden_array("rmsnorm", f"{name}/out_plain"), dt).float().numpy()
        np.testing.assert_allclose(out, want, atol=tol, rtol=tol)
        np.testing.assert_allclose(plain, want_plain, atol=tol, rtol=tol)


def test_bf16_rounding_is_round_to_nearest_even():
    x = torch.randn(10000) * 10
    x = torch.cat([x, torch.tensor([0.0, -0.0, float("inf"), float("-inf"), 1e-40, 3.0e38])])
    got = oracle.round_to(x.numpy(), "bf16")
    want = x.to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(got, want)
    assert np.isnan(oracle.round_to(np.array([np.nan], np.float32), "bf16")).all()
    bits = oracle.f32_to_bf16_bits(x.numpy())
    np.testing.assert_array_equal(bits, x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))


def test_oracle_zero_length_sequence_gives_zeros():
    """kernel-lab's reference returns zeros for an empty sequence (empty einsum)."""
    q = np.ones((2, 2, 8), np.float32)
    k = np.ones((2, 16, 1, 8), np.float32)
    bt = np.array([[0], [1]], np.int32)
    out = oracle.paged_decode_attention(q, k, k, bt, np.array([0, 5], np.int32))
    assert (out[0] == 0).all() and np.allclose(out[1], 1.0)


def test_decode_bytes_model():
    """The roofline's algorithmic bytes (kernel-lab tests/test_roofline.py:23-26)."""
    assert oracle.decode_bytes([10, 20], 4, 2, 8, 2) == 2 * 30 * 2 * 8 * 2 + 2 * 2 * 4 * 8 * 2
    # Config 3 headline: batch 64, context 4096, Llama-3-8B heads, bf16.
    assert oracle.decode_bytes([4096] * 64, 32, 8, 128, 2) == 1_074_790_400


def test_append_oracle_rebuilds_the_fixture_pool_token_by_token():
    """Appending every token of every sequence, in order, through the append oracle fills the
    same pages as kernel-lab's fixture builder (kv_cache.py:33-80, restated in this package's
    build_paged_kv); spare pages are untouched, bad pages and padding are reported / skipped."""
    import torch

    from kernel_lab.kv_cache import build_paged_kv, pages_for

    lens = [1, 15, 16, 17, 40]
    keys = [torch.randn(n, 2, 8) for n in lens]
    values = [torch.randn(n, 2, 8) for n in lens]
    kv = build_paged_kv(keys, values, page_size=16, poison=0.0)
    k = np.zeros_like(kv.k_cache.numpy())
    v = np.zeros_like(kv.v_cache.numpy())
    bt = kv.block_table.numpy()
    for t in range(max(lens)):
        pos = np.array([t if t < n else -1 for n in lens], np.int32)
        kn = np.stack([keys[b][min(t, n - 1)].numpy() for b, n in enumerate(lens)])
        vn = np.stack([values[b][min(t, n - 1)].numpy() for b, n in enumerate(lens)])
        k, v, status = oracle.paged_kv_append(k, v, kn, vn, bt, pos)
        assert status == 0
    np.testing.assert_array_equal(k, kv.k_cache.numpy())
    np.testing.assert_array_equal(v, kv.v_cache.numpy())
    assert [pages_for(n, 16) for n in lens] == [1, 1, 1, 2, 3]

    bad = bt.copy()
    bad[0, 0] = kv.num_pages  # out of the pool
    k2, _, status = oracle.paged_kv_append(k, v, np.ones((5, 2, 8), np.float32), np.ones((5, 2, 8), np.float32), bad,
                                           np.array([0, -1, -1, -1, 16 * bt.shape[1]], np.int32))
    assert status == oracle.KL_STATUS_BAD_PAGE
    np.testing.assert_array_equal(k2, k)  # both writes skipped


def test_e4m3_codec_is_pinned_to_torch_float8():
    """The oracle's e4m3 codec against torch.float8_e4m3fn: every code decodes to the same value;
    encoding rounds to nearest-even exactly as torch wherever torch's result is finite (|x| <
    464); beyond that the oracle saturates to +-448 (the kernels' saturate-finite rounding,
    which torch's cast does not do) and NaN stays NaN."""
    import torch

    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(oracle.e4m3_decode(codes), want)
    rng = np.random.default_rng(7)
    x = np.concatenate([rng.standard_normal(50_000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0, 200.0)])
    x = np.concatenate([x, oracle.E4M3_VALUES[np.isfinite(oracle.E4M3_VALUES)]])
    x = x[np.abs(x) < 464]
    torch_codes = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(oracle.e4m3_encode(x), torch_codes)
    sat = oracle.e4m3_decode(oracle.e4m3_encode(np.array([470.0, 1e6, -1e6, np.nan], np.float32)))
    assert sat[:3].tolist() == [448.0, 448.0, -448.0] and np.isnan(sat[3])


def test_fp8_append_oracle_quantises_then_scatters():
    hkv, d = 2, 8
    k_codes = np.zeros((3, 4, hkv, d), np.uint8)
    bt = np.array([[2, 0], [1, 0]], np.int32)
    k_new = np.linspace(-3, 3, 2 * hkv * d, dtype=np.float32).reshape(2, hkv, d)
    k_new[0, 1, 3] = 7.0  # 7 / 0.01 = 700 > 448: saturates
    scale = np.array([0.5, 0.01], np.float32)
    k2, v2, status = oracle.paged_kv_append_fp8(k_codes, k_codes, k_new, k_new, scale, scale, bt,
                                                np.array([5, -1], np.int32))
    assert status == 0
    # position 5 of sequence 0: page bt[0, 1] = 0, slot 1; one head-1 value saturates
    got = oracle.e4m3_decode(k2[0, 1]) * scale[:, None]
    np.testing.assert_allclose(got[0], k_new[0, 0], rtol=2**-3)
    assert oracle.e4m3_decode(k2[0, 1, 1])[3] == 448.0
    assert (k2[1:] == 0).all() and (k2[0, 0] == 0).all()


# ---------------------------------------------------------------- cascade (shared prefix)
#
# kernel-lab has no cascade, so the cascade oracle is pinned to the pinned decode oracle: with
# page-aligned prefixes it must equal plain decode over the concatenated block tables bit for bit,
# and with ragged prefixes it must equal a per-token loop written independently of both.


def _cascade_case(group_sizes, prefix_lens, seq_lens, hq=8, hkv=2, d=32, page=8, seed=3):
    from kernel_lab.kv_cache import random_cascade_problem

    q, kv = random_cascade_problem(
        group_sizes, prefix_lens, seq_lens, hq, hkv, d, page, dtype=torch.float32, device="cpu", seed=seed
    )
    return q.numpy(), kv


def _np(kv, name):
    return getattr(kv, name).numpy()


def _oracle_cascade(q, kv, **kw):
    return oracle.paged_decode_attention_cascade(
        q, _np(kv, "k_cache"), _np(kv, "v_cache"), _np(kv, "prefix_block_table"), _np(kv, "prefix_lens"),
        _np(kv, "prefix_indptr"), _np(kv, "block_table"), _np(kv, "seq_lens"), **kw
    )


def test_cascade_oracle_equals_plain_decode_over_concatenated_tables():
    q, kv = _cascade_case([3, 1, 0, 4], [16, 0, 24, 40], [5, 0, 9, 17, 1, 8, 0, 30])
    table, lens = kv.concatenated_tables()
    want = oracle.paged_decode_attention(q, _np(kv, "k_cache"), _np(kv, "v_cache"), table.numpy(), lens.numpy())
    got = _oracle_cascade(q, kv)
    assert np.array_equal(got, want)


def test_cascade_oracle_ragged_prefix_matches_token_loop():
    q, kv = _cascade_case([2, 3], [13, 7], [3, 0, 11, 6, 2], seed=5)
    k_cache, v_cache = _np(kv, "k_cache"), _np(kv, "v_cache")
    page = kv.page_size
    indptr = kv.prefix_indptr.tolist()
    hq, d = q.shape[1], q.shape[2]
    g = hq // k_cache.shape[2]
    want = np.zeros_like(q)
    for p in range(len(indptr) - 1):
        for b in range(indptr[p], indptr[p + 1]):
            rows = [(int(kv.prefix_block_table[p, t // page]), t % page) for t in range(int(kv.prefix_lens[p]))]
            rows += [(int(kv.block_table[b, t // page]), t % page) for t in range(int(kv.seq_lens[b]))]
            for h in range(hq):
                if not rows:
                    continue
                s = np.array([float(np.dot(q[b, h], k_cache[pg, sl, h // g])) for pg, sl in rows]) * d**-0.5
                w = np.exp(s - s.max())
                w /= w.sum()
                want[b, h] = sum(wi * v_cache[pg, sl, h // g] for wi, (pg, sl) in zip(w, rows))
    got = _oracle_cascade(q, kv)
    np.testing.assert_allclose(got, want, atol=2e-6, rtol=1e-5)


def test_cascade_oracle_ignores_prefixes_when_groups_do_not_partition_the_batch():
    q, kv = _cascade_case([2, 2], [16, 8], [4, 5, 6, 7])
    kv.prefix_indptr = torch.tensor([0, 3, 2], dtype=torch.int32)  # decreasing
    got = _oracle_cascade(q, kv)
    want = oracle.paged_decode_attention(q, _np(kv, "k_cache"), _np(kv, "v_cache"), _np(kv, "block_table"),
                                         _np(kv, "seq_lens"))
    assert np.array_equal(got, want)


def test_cascade_builder_tables_are_disjoint_and_spares_poisoned():
    _, kv = _cascade_case([2, 1], [17, 9], [4, 0, 23])
    page = kv.page_size
    used = set()
    for p, n in enumerate(kv.prefix_lens.tolist()):
        used |= set(kv.prefix_block_table[p, : -(-n // page)].tolist())
    for b, n in enumerate(kv.seq_lens.tolist()):
        row = set(kv.block_table[b, : -(-n // page)].tolist())
        assert not (row & used)
        used |= row
    spare = sorted(set(range(kv.k_cache.shape[0])) - used)
    assert spare and torch.isnan(kv.k_cache[spare]).all() and torch.isnan(kv.v_cache[spare]).all()
