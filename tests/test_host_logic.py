"""Host-side logic without a GPU: roofline model, fixture builders, bench contract."""

from __future__ import annotations

import json
import math
import subprocess
import sys

import numpy as np
import pytest
import torch

from tests.conftest import REPO


def test_roofline_byte_model_matches_kernel_lab():
    """kernel-lab tests/test_roofline.py:9-26 counts, and the headline's bytes."""
    from kernel_lab import roofline

    w = roofline.rms_norm_work(rows=2, hidden=8, elem_bytes=2, fused_residual=True)
    assert w.bytes == 2 * 8 * 2 * 4 + 8 * 2
    assert roofline.rms_norm_work(2, 8, 2, False).bytes == 2 * 8 * 2 * 2 + 8 * 2
    work = roofline.decode_attention_work([10, 20], num_q_heads=4, num_kv_heads=2, head_dim=8, elem_bytes=2)
    assert work.bytes == 2 * 30 * 2 * 8 * 2 + 2 * 2 * 4 * 8 * 2
    assert work.flops == 4 * 30 * 4 * 8
    head = roofline.decode_attention_work([4096] * 64, 32, 8, 128, 2)
    assert head.bytes == 1_074_790_400
    assert 3.5 < roofline.decode_attention_work([4096] * 8, 32, 8, 128, 2).intensity < 4.5
    assert roofline.rms_norm_work(4096, 8192, 2, True).bytes == 268_451_840


def test_measured_peaks_loader(tmp_path):
    from kernel_lab import roofline

    p = tmp_path / "peaks.json"
    p.write_text(json.dumps({"hbm_gbs": 6500.0, "bf16_tflops": 1600.0}))
    pk = roofline.measured_peaks(p)
    assert pk.hbm_gbps == 6500.0 and pk.source == "measured"
    assert roofline.measured_peaks(tmp_path / "missing.json").source == "fallback"


def test_builder_poisons_spares_zeroes_tails_and_shuffles():
    from kernel_lab.kv_cache import build_paged_kv, pages_for

    keys = [torch.randn(n, 2, 8) for n in (5, 33)]
    values = [torch.randn(n, 2, 8) for n in (5, 33)]
    kv = build_paged_kv(keys, values, page_size=16)
    used = set(kv.block_table[0, :1].tolist()) | set(kv.block_table[1, :3].tolist())
    spare = sorted(set(range(kv.num_pages)) - used)
    assert len(spare) == 3 and torch.isnan(kv.k_cache[spare]).all() and torch.isnan(kv.v_cache[spare]).all()
    assert (kv.k_cache[kv.block_table[0, 0], 5:] == 0).all()  # tail of a partial page
    for b, k in enumerate(keys):
        n = k.shape[0]
        pages = kv.block_table[b, : pages_for(n, 16)].long()
        torch.testing.assert_close(kv.k_cache[pages].reshape(-1, 2, 8)[:n], k)
    assert kv.block_table[1].tolist() != sorted(kv.block_table[1].tolist())
    with pytest.raises(ValueError):
        build_paged_kv([torch.randn(0, 1, 8)], [torch.randn(0, 1, 8)], page_size=16)


def test_serving_pool_builder_and_head_shards():
    """random_paged_pool: valid tables, NaN spares, zero tails; a KV-head slice equals the
    same heads of the full pool (so the union of shards is the unsharded problem)."""
    from kernel_lab.kv_cache import random_paged_pool

    lens = [1, 17, 40]
    q, kv = random_paged_pool(lens, 8, 4, 16, 16, dtype=torch.float32, device="cpu", seed=5)
    need = [math.ceil(n / 16) for n in lens]
    ids = torch.cat([kv.block_table[b, :n] for b, n in enumerate(need)])
    assert len(set(ids.tolist())) == sum(need) and int(ids.max()) < kv.num_pages
    spare = sorted(set(range(kv.num_pages)) - set(ids.tolist()))
    assert torch.isnan(kv.k_cache[spare]).all()
    assert (kv.v_cache[kv.block_table[1, 1], 1:] == 0).all()
    q2, kv2 = random_paged_pool(lens, 8, 4, 16, 16, dtype=torch.float32, device="cpu", seed=5, kv_head_slice=(2, 4))
    np.testing.assert_array_equal(q2.numpy(), q[:, 4:8].numpy())
    np.testing.assert_array_equal(kv2.k_cache[ids].numpy(), kv.k_cache[ids][:, :, 2:4].numpy())


def test_bench_reference_arm_prints_the_contract_line():
    proc = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1",
         "--ctx", "512"],
        capture_output=True, text=True, timeout=600,
    )
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["steps"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
