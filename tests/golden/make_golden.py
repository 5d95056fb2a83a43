"""Generate the golden vectors in this directory from the reference implementation itself.

Run once, where the reference source tree is available (it is not on GPU boxes):

    python tests/golden/make_golden.py /path/to/kernel-lab

It imports the reference's ``kernel_lab.reference`` (PyTorch fp32 CPU math) and
``kernel_lab.kv_cache`` (seeded fixture builder), builds the cases below exactly
as the reference's tests build theirs, and stores per case:

* ``<case>/in_sha256``: SHA-256 of every input tensor's raw bytes, as the
  reference's builder produced it (spare pages poisoned with 1e4). The tests
  rebuild the inputs with this repository's ``kernel_lab.kv_cache`` (poison=1e4)
  and must reproduce these hashes, which pins the fixture builder.
* ``<case>/out...``: the reference's outputs (full arrays when small; for the
  4096-row RMSNorm cases a SHA-256 of the bit-exact residual and sampled rows of
  the normalised output).

Everything lands in ``decode.npz``, ``rmsnorm.npz`` and ``index.json``.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def sha(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def decode_cases():
    cases = []
    # Triton-suite shapes (tests/test_paged_attention.py:11-14): D=32, page-boundary lengths.
    for dt in ("f32", "f16", "bf16"):
        for hq, hkv in ((4, 4), (8, 2), (8, 1)):
            cases.append(dict(name=f"tri_{hq}_{hkv}_{dt}", lens=[1, 15, 16, 17, 33, 70], hq=hq, hkv=hkv, d=32, p=16, dt=dt))
    # CUDA-suite shapes (tests/test_cuda_kernels.py:44-53).
    for dt in ("f32", "f16", "bf16"):
        for hq, hkv in ((8, 8), (16, 4), (8, 1), (32, 8)):
            cases.append(dict(name=f"cu_{hq}_{hkv}_128_{dt}", lens=[1, 3, 16, 17, 300, 1025], hq=hq, hkv=hkv, d=128, p=16, dt=dt))
    for d in (64, 256):
        cases.append(dict(name=f"cu_32_8_{d}_bf16", lens=[1, 3, 16, 17, 300, 1025], hq=32, hkv=8, d=d, p=16, dt="bf16"))
        cases.append(dict(name=f"cu_8_1_{d}_f16", lens=[1, 3, 16, 17, 300, 1025], hq=8, hkv=1, d=d, p=16, dt="f16"))
    # Page and head sizes (tests/test_paged_attention.py:47-53).
    for p in (16, 32):
        for d in (32, 64):
            cases.append(dict(name=f"page_{p}_{d}", lens=[3, 50], hq=4, hkv=2, d=d, p=p, dt="f32"))
    cases.append(dict(name="page_8_128_bf16", lens=[3, 50, 129], hq=8, hkv=2, d=128, p=8, dt="bf16"))
    cases.append(dict(name="page_64_128_bf16", lens=[3, 50, 129], hq=8, hkv=2, d=128, p=64, dt="bf16"))
    # Custom scale (tests/test_paged_attention.py:72-78).
    cases.append(dict(name="scale_005", lens=[12], hq=2, hkv=2, d=32, p=16, dt="f32", scale=0.05))
    # batch 4, length 512, Llama-3-8B heads, fp16.
    cases.append(dict(name="cfg1", lens=[512] * 4, hq=32, hkv=8, d=128, p=16, dt="f16"))
    # Config 3 samples (bf16, Llama-3-8B heads).
    cases.append(dict(name="cfg3_b1_512", lens=[512], hq=32, hkv=8, d=128, p=16, dt="bf16"))
    cases.append(dict(name="cfg3_b8_512", lens=[512] * 8, hq=32, hkv=8, d=128, p=16, dt="bf16"))
    # Config 4 samples: ragged lengths at and around multiples of 16; MQA / GQA / MHA.
    ragged = [1, 15, 16, 17, 255, 256, 257, 1000]
    for hq, hkv in ((32, 1), (32, 8), (32, 32)):
        cases.append(dict(name=f"cfg4_{hq}_{hkv}", lens=ragged, hq=hq, hkv=hkv, d=128, p=16, dt="bf16"))
    # Config 5 sample: Llama-3-70B heads.
    cases.append(dict(name="cfg5_sample", lens=[300, 77], hq=64, hkv=8, d=128, p=16, dt="bf16"))
    return cases


def rms_cases():
    cases = []
    for dt in ("f32", "f16", "bf16"):
        for shape in ((1, 16), (3, 100), (4, 256), (2, 3, 128), (7, 1000)):
            cases.append(dict(name=f"t_{'x'.join(map(str, shape))}_{dt}", shape=list(shape), dt=dt, eps=1e-6))
    for rows in (1, 16, 256, 4096):
        for hidden in (4096, 8192):
            cases.append(dict(name=f"cfg2_{rows}x{hidden}", shape=[rows, hidden], dt="bf16", eps=1e-5))
    return cases


def make(shape, dtype, seed=0):
    """Input protocol of tests/test_rmsnorm.py:14-19."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g).to(dtype=dtype)
    r = torch.randn(*shape, generator=g).to(dtype=dtype)
    w = (1 + 0.1 * torch.randn(shape[-1], generator=g)).to(dtype=dtype)
    return x, r, w


def main(ref_root: str) -> None:
    sys.dont_write_bytecode = True
    sys.path.insert(0, ref_root)
    from kernel_lab import reference  # the reference's own oracle
    from kernel_lab.kv_cache import build_paged_kv, random_decode_problem

    index = {"decode": [], "rmsnorm": [], "generator": "tests/golden/make_golden.py", "torch": torch.__version__}
    arrays: dict[str, np.ndarray] = {}

    for c in decode_cases():
        dtype = DT[c["dt"]]
        q, kv, _, _ = random_decode_problem(c["lens"], c["hq"], c["hkv"], c["d"], c["p"], dtype=dtype, seed=0)
        out = reference.paged_decode_attention(
            q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, scale=c.get("scale")
        )
        c["in_sha256"] = {
            "q": sha(q),
            "k_cache": sha(kv.k_cache),
            "v_cache": sha(kv.v_cache),
            "block_table": sha(kv.block_table),
            "seq_lens": sha(kv.seq_lens),
        }
        c["num_pages"] = int(kv.k_cache.shape[0])
        arrays[f"{c['name']}/out"] = to_np(out)
        index["decode"].append(c)

    # Known answer (tests/test_paged_attention.py:81-91): one key far more aligned than the
    # rest, values v[t] = t, so the output is 13.0 everywhere.
    d = 32
    keys = [torch.zeros(20, 1, d)]
    values = [torch.arange(20, dtype=torch.float32)[:, None, None].expand(20, 1, d).clone()]
    keys[0][13, 0, 0] = 100.0
    kv = build_paged_kv(keys, values, page_size=16)
    q = torch.zeros(1, 1, d)
    q[0, 0, 0] = 1.0
    out = reference.paged_decode_attention(q, kv.k_cache, kv.v_cache, kv.block_table, kv.seq_lens, scale=1.0)
    index["onehot"] = {
        "in_sha256": {"k_cache": sha(kv.k_cache), "v_cache": sha(kv.v_cache), "block_table": sha(kv.block_table)},
    }
    arrays["onehot/out"] = to_np(out)

    for c in rms_cases():
        dtype = DT[c["dt"]]
        x, r, w = make(c["shape"], dtype)
        out_plain = reference.rms_norm(x, w, c["eps"])
        out, new_res = reference.fused_add_rms_norm(x, r, w, c["eps"])
        c["in_sha256"] = {"x": sha(x), "residual": sha(r), "weight": sha(w)}
        c["residual_out_sha256"] = sha(new_res)
        rows = int(np.prod(c["shape"][:-1]))
        if rows * c["shape"][-1] <= 1 << 13:
            arrays[f"{c['name']}/out"] = to_np(out)
            arrays[f"{c['name']}/out_plain"] = to_np(out_plain)
            arrays[f"{c['name']}/residual_out"] = to_np(new_res)
        else:
            sample = sorted({0, rows // 2, rows - 1})
            c["sample_rows"] = sample
            h = c["shape"][-1]
            arrays[f"{c['name']}/out_rows"] = to_np(out.reshape(rows, h)[sample])
            arrays[f"{c['name']}/out_plain_rows"] = to_np(out_plain.reshape(rows, h)[sample])
        index["rmsnorm"].append(c)

    dec = {k: v for k, v in arrays.items() if not k.startswith(("t_", "cfg2_"))}
    rms = {k: v for k, v in arrays.items() if k.startswith(("t_", "cfg2_"))}
    np.savez_compressed(HERE / "decode.npz", **dec)
    np.savez_compressed(HERE / "rmsnorm.npz", **rms)
    (HERE / "index.json").write_text(json.dumps(index, indent=1) + "\n")
    print(f"wrote {len(dec)} decode arrays, {len(rms)} rmsnorm arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference source root>")
    main(sys.argv[1])
