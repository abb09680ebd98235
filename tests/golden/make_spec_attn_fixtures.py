"""Generate golden vectors for the speculative-verification attention by running the reference's own kernels.

Run in the build container (the one that has the reference checkout):

    python tests/golden/make_spec_attn_fixtures.py --reference <path to the qwen-a100-fastpath checkout>

It imports ``qwen_fastpath.spec_attn`` from ``<reference>/plugin`` and calls ``gqa_packed_spec_attention``
(plugin/qwen_fastpath/spec_attn.py:139-173) unmodified, i.e. the Triton kernels ``_prefix_split_kernel`` and
``_suffix_combine_kernel`` (:17-136), under Triton's CPU interpreter, twice per case:

* ``out_f32``: query, cache and output held in fp32 (bf16-valued inputs).  The kernels then run in fp32 throughout
  (``p.to(v.dtype)`` keeps fp32), which checks the algorithm -- split arithmetic, masks, the log-sum-exp merge --
  against ``oracle.spec_attn_oracle.attention`` to fp32 rounding.
* ``out_bf16``: bf16 tensors, with the interpreter's bf16 conversions and ``tl.dot`` replaced by exact ones (the
  fixes of ``make_fixtures.py``; the interpreter mishandles bf16 otherwise): the reference's own bf16 arithmetic
  (P rounded to bf16 before P V, bf16 output), the target of the GPU parity test.

Cases cover an empty prefix (context 0), a request shorter than Q, several requests of different lengths, shuffled
pages, one and several splits, G = 1 / 3 / 6, head sizes 64 / 128 / 256.  Inputs come from
``oracle.spec_attn_oracle.make_case`` (numpy RandomState streams); their sha256 is stored so that a drift in the
generator is detected.  Nothing here runs on the GPU box: only the committed ``.npz`` travels.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))
from oracle import spec_attn_oracle as sao  # noqa: E402

# (name, seed, num_reqs, Q, H, HKV, D, page, lens, num_splits, min_chunk, block_n)
CASES = [
    ("ctx100_q3", 1, 1, 3, 6, 2, 64, 32, [103], 4, 32, 16),
    ("two_reqs_splits", 2, 2, 4, 8, 2, 64, 16, [304, 297], 8, 32, 16),
    ("empty_prefix", 3, 1, 3, 6, 2, 64, 16, [3], 4, 32, 16),
    ("shorter_than_q", 4, 1, 3, 6, 2, 64, 16, [1], 4, 32, 16),
    ("three_reqs_g1_d128", 5, 3, 2, 2, 2, 128, 32, [70, 1, 45], 4, 32, 16),
    ("g6_d256_q5", 6, 1, 5, 6, 1, 256, 48, [517], 8, 64, 32),
    ("page800_two", 7, 2, 3, 6, 1, 64, 800, [850, 843], 16, 32, 32),
]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def run(fn, q_bits, kv_bits, bt, lens, Q, HKV, D, scale, ns, mc, bn, dtype):
    q = torch.from_numpy(q_bits.view(np.int16)).view(torch.bfloat16).to(dtype)
    kv = torch.from_numpy(kv_bits.view(np.int16)).view(torch.bfloat16).to(dtype)
    kc, vc = kv.transpose(1, 2).split(D, dim=-1)
    out = torch.zeros_like(q)
    fn(q, kc, vc, out, torch.from_numpy(lens), torch.from_numpy(bt), len(lens), Q, HKV, scale, num_splits=ns,
       min_chunk=mc, block_n=bn)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the qwen-a100-fastpath checkout")
    ap.add_argument("--out", default=str(HERE / "spec_attn_reference.npz"))
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "plugin"))
    from qwen_fastpath.spec_attn import gqa_packed_spec_attention as ref  # the reference, unmodified
    from make_fixtures import fix_triton_interpreter_bf16

    arrays = {}
    names = []
    for name, seed, B, Q, H, HKV, D, page, lens, ns, mc, bn in CASES:
        q_bits, kv_bits, bt, lens_a = sao.make_case(seed, B, Q, H, HKV, D, page, lens)
        scale = D ** -0.5
        out32 = run(ref, q_bits, kv_bits, bt, lens_a, Q, HKV, D, scale, ns, mc, bn, torch.float32)
        arrays[f"{name}/q"] = q_bits
        arrays[f"{name}/kv"] = kv_bits
        arrays[f"{name}/block_table"] = bt
        arrays[f"{name}/seq_lens"] = lens_a
        arrays[f"{name}/params"] = np.array([B, Q, H, HKV, D, page, seed], np.int64)
        arrays[f"{name}/scale"] = np.array([scale], np.float64)
        arrays[f"{name}/out_f32"] = out32.numpy()
        arrays[f"{name}/input_sha256"] = np.frombuffer(sha(q_bits, kv_bits, bt, lens_a).encode(), np.uint8)
        names.append(name)
        print(f"{name}: f32 done", flush=True)
    fix_triton_interpreter_bf16()
    for name, seed, B, Q, H, HKV, D, page, lens, ns, mc, bn in CASES:
        q_bits, kv_bits, bt, lens_a = (arrays[f"{name}/q"], arrays[f"{name}/kv"], arrays[f"{name}/block_table"],
                                       arrays[f"{name}/seq_lens"])
        out16 = run(ref, q_bits, kv_bits, bt, lens_a, Q, HKV, D, D ** -0.5, ns, mc, bn, torch.bfloat16)
        arrays[f"{name}/out_bf16"] = out16.view(torch.int16).numpy().view(np.uint16).copy()
        print(f"{name}: bf16 done", flush=True)
    arrays["cases"] = np.array(names)
    np.savez_compressed(args.out, **arrays)
    print("wrote", args.out, os.path.getsize(args.out), "bytes")


if __name__ == "__main__":
    main()
