"""Generate golden vectors by running the reference plugin's own code on the CPU.

Run in the build container (the one that has the reference checkout):

    python tests/golden/make_fixtures.py --reference <path to the qwen-a100-fastpath checkout>

It imports ``qwen_fastpath`` from ``<reference>/plugin`` and executes, unmodified:

* ``w8a16_mm`` / ``pick_config`` (plugin/qwen_fastpath/w8a16.py:58-83), i.e. the Triton kernel
  ``_w8a16_kernel`` (w8a16.py:15-44) under ``TRITON_INTERPRET=1``;
* ``patch_int8_linear`` (plugin/qwen_fastpath/patches.py:72-116): the ``qf_int8_linear`` op and the
  patched ``apply_weights`` against a stand-in ``CutlassInt8ScaledMMLinearKernel``;
* ``patch_draft_lm_head`` (patches.py:119-189): the load-time int8 quantizer, ``compute_logits`` and
  ``get_top_tokens`` against stand-in ``Qwen3_5MTP`` / ``MTPSpeculator`` classes.

Triton's CPU interpreter (triton 3.6) mishandles bfloat16: an int -> bf16 cast stores the integer value as
the raw uint16 pattern, ``tl.dot`` multiplies raw bf16 bit patterns as integers, and its fp32 -> bf16
rounding does not carry into the exponent.  Those three interpreter functions are replaced here by exact
conversions (torch's bf16 conversion, round to nearest even); the kernel's own tiling, masking, split-K
fp32 atomics, scale epilogue and output rounding are what run.  ``tl.dot`` then accumulates in fp32 as the
tensor-core path does (summation order differs, as it does between GPUs).

Inputs come from ``oracle.w8a16_oracle.make_inputs`` (numpy RandomState streams, frozen across
versions); the fixture stores their sha256 so a drift in the generator is detected, plus the reference's
outputs.  Nothing here runs on the GPU box: only the committed ``.npz`` / ``.json`` travel.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
from oracle import w8a16_oracle as orc  # noqa: E402

# (N, K, M, x_row_stride) -- ragged N, split-K > 1, strided x rows, K = 2176 (17408 / 8), M in 1..16
GEMM_CASES = [
    (64, 256, 1, None),
    (100, 512, 3, None),
    (1000, 1024, 5, 1040),
    (2048, 2176, 16, None),
    (8192, 512, 8, None),
    (320, 1024, 12, None),
    (96, 128, 2, None),
    (5120, 512, 4, None),
]
PICK_CONFIG_SHAPES = [
    (5120, 5120), (10240, 5120), (5120, 8192), (34816, 5120), (5120, 17408), (151936, 5120),
    (34816, 5120), (5120, 17408), (16384, 5120), (5120, 6144), (14336, 5120), (248320, 5120),
    (1280, 5120), (5120, 2176), (18992, 5120), (64, 100), (96, 128),
]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def bits_to_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bf16_to_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


# ----------------------------------------------------------------------------------------------
# Triton interpreter bf16 fixes
# ----------------------------------------------------------------------------------------------
def fix_triton_interpreter_bf16() -> None:
    import triton.language as tl
    from triton.runtime import interpreter as itp

    builder = itp.InterpreterBuilder
    orig_cast = builder.cast_impl
    orig_fp_to_fp = builder.create_fp_to_fp
    orig_dot = builder.create_dot

    def as_f32(handle) -> np.ndarray:
        if handle.dtype.scalar == tl.bfloat16:
            return (handle.data.astype(np.uint32) << 16).view(np.float32)
        return handle.data.astype(np.float32)

    def to_bf16_bits(vals: np.ndarray) -> np.ndarray:
        t = torch.from_numpy(np.ascontiguousarray(vals, dtype=np.float32)).to(torch.bfloat16)
        return t.view(torch.int16).numpy().view(np.uint16).reshape(vals.shape)

    def convert(self, src, dst_type, fallback, *args):
        s, d = src.dtype.scalar, dst_type.scalar
        if d == tl.bfloat16 and s != tl.bfloat16:
            return itp.TensorHandle(to_bf16_bits(as_f32(src)), d)
        if s == tl.bfloat16 and d != tl.bfloat16:
            return itp.TensorHandle(as_f32(src).astype(itp._get_np_dtype(dst_type)), d)
        return fallback(self, src, dst_type, *args)

    def cast_impl(self, src, dst_type):
        return convert(self, src, dst_type, orig_cast)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        return convert(self, src, dst_type, orig_fp_to_fp, rounding_mode)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            out = np.matmul(as_f32(a), as_f32(b), dtype=np.float32) + d.data
            return itp.TensorHandle(out.astype(d.data.dtype), d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    builder.cast_impl = cast_impl
    builder.create_fp_to_fp = create_fp_to_fp
    builder.create_dot = create_dot


# ----------------------------------------------------------------------------------------------
# stand-ins for the vLLM classes the patches target
# ----------------------------------------------------------------------------------------------
class FallbackTaken(RuntimeError):
    pass


def install_fake_vllm():
    lib = torch.library.Library("vllm", "FRAGMENT")  # noqa: the op lives as long as this object

    def mod(name):
        m = types.ModuleType(name)
        sys.modules[name] = m
        parent, _, child = name.rpartition(".")
        if parent:
            setattr(sys.modules[parent], child, m)
        return m

    for name in ["vllm", "vllm.model_executor", "vllm.model_executor.kernels",
                 "vllm.model_executor.kernels.linear", "vllm.model_executor.kernels.linear.scaled_mm",
                 "vllm.model_executor.kernels.linear.scaled_mm.cutlass", "vllm.utils",
                 "vllm.utils.torch_utils", "vllm.model_executor.models",
                 "vllm.model_executor.models.qwen3_5_mtp", "vllm.v1", "vllm.v1.worker", "vllm.v1.worker.gpu",
                 "vllm.v1.worker.gpu.spec_decode", "vllm.v1.worker.gpu.spec_decode.mtp",
                 "vllm.v1.worker.gpu.spec_decode.mtp.speculator", "vllm._custom_ops"]:
        mod(name)

    ops = sys.modules["vllm._custom_ops"]

    def scaled_int8_quant(*a, **k):
        raise FallbackTaken("scaled_int8_quant")

    ops.scaled_int8_quant = scaled_int8_quant
    ops.cutlass_scaled_mm = scaled_int8_quant

    class CutlassInt8ScaledMMLinearKernel:
        def _get_layer_params(self, layer):
            return layer.weight, layer.weight_scale, layer.input_scale, None, None

        def apply_weights(self, layer, x, bias=None):
            raise FallbackTaken("orig_apply")

    sys.modules["vllm.model_executor.kernels.linear.scaled_mm.cutlass"].CutlassInt8ScaledMMLinearKernel = \
        CutlassInt8ScaledMMLinearKernel

    def direct_register_custom_op(op_name, op_func, mutates_args=None, fake_impl=None, **_):
        schema = torch.library.infer_schema(op_func, mutates_args=mutates_args or [])
        lib.define(op_name + schema)
        lib.impl(op_name, op_func, "CPU")

    sys.modules["vllm.utils.torch_utils"].direct_register_custom_op = direct_register_custom_op

    class Qwen3_5MTP:
        def compute_logits(self, hidden_states, spec_step_idx=0):
            raise FallbackTaken("orig_compute_logits")

        def get_top_tokens(self, hidden_states):
            raise FallbackTaken("orig_get_top_tokens")

    sys.modules["vllm.model_executor.models.qwen3_5_mtp"].Qwen3_5MTP = Qwen3_5MTP

    class MTPSpeculator:
        def load_draft_model(self, target_model, target_attn_layer_names):
            return self.draft

    sys.modules["vllm.v1.worker.gpu.spec_decode.mtp.speculator"].MTPSpeculator = MTPSpeculator
    return lib, CutlassInt8ScaledMMLinearKernel, Qwen3_5MTP, MTPSpeculator


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the qwen-a100-fastpath checkout")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()

    fix_triton_interpreter_bf16()
    keep = install_fake_vllm()
    _lib, Kernel, MTP, Spec = keep
    sys.path.insert(0, str(Path(args.reference) / "plugin"))
    import qwen_fastpath  # noqa: F401
    from qwen_fastpath import patches
    from qwen_fastpath.w8a16 import SMALL_M, pick_config, w8a16_mm

    meta = {"generator": "tests/golden/make_fixtures.py", "torch": torch.__version__, "numpy": np.__version__,
            "small_m": SMALL_M, "gemm": [], "linear": [], "head": {}, "pick_config": {}}
    arrays = {}

    for (N, K) in PICK_CONFIG_SHAPES:
        meta["pick_config"][f"{N},{K}"] = pick_config(N, K)

    # ---- w8a16_mm --------------------------------------------------------------------------
    for i, (N, K, M, ldx) in enumerate(GEMM_CASES):
        seed = 1000 + i
        x_bits, W, s = orc.make_inputs(seed, M, N, K, x_row_stride=ldx)
        cfg = pick_config(N, K)
        x_t = bits_to_bf16(x_bits)[:, :K]          # row stride ldx, unit column stride
        y = w8a16_mm(x_t, torch.from_numpy(W).t(), torch.from_numpy(s), cfg, torch.bfloat16)
        arrays[f"gemm{i}_y"] = bf16_to_bits(y)
        meta["gemm"].append({"case": i, "seed": seed, "N": N, "K": K, "M": M, "ldx": ldx or K,
                             "cfg": cfg, "inputs_sha256": sha(x_bits, W, s)})
        print(f"gemm case {i}: N={N} K={K} M={M} ldx={ldx} cfg={cfg}", flush=True)

    # ---- qf_int8_linear through the patched apply_weights ------------------------------------
    patches.patch_int8_linear()
    kern = Kernel()
    for j, (lead, N, K, with_bias) in enumerate([((2, 3), 384, 512, True), ((5,), 640, 256, False),
                                                  ((1,), 200, 1024, True), ((17,), 128, 256, False)]):
        M = int(np.prod(lead))
        seed = 2000 + j
        x_bits, W, s = orc.make_inputs(seed, M, N, K)
        bias_bits = orc.make_bias(seed + 500, N) if with_bias else None
        layer = types.SimpleNamespace(weight=torch.from_numpy(W).t(),                       # [K, N], stride (1, K)
                                      weight_scale=torch.from_numpy(s).reshape(N, 1),     # [N, 1] fp32
                                      input_scale=None)
        x = bits_to_bf16(x_bits).reshape(*lead, K)
        b = bits_to_bf16(bias_bits) if with_bias else None
        entry = {"case": j, "seed": seed, "lead": list(lead), "N": N, "K": K, "bias": with_bias,
                 "bias_seed": seed + 500 if with_bias else None, "inputs_sha256": sha(x_bits, W, s)}
        try:
            y = kern.apply_weights(layer, x, b)
            arrays[f"linear{j}_y"] = bf16_to_bits(y)
            entry["path"] = "w8a16"
            entry["out_shape"] = list(y.shape)
        except FallbackTaken as e:
            entry["path"] = f"fallback:{e}"
        meta["linear"].append(entry)
        print(f"linear case {j}: {entry['path']}", flush=True)

    # ---- draft lm_head ----------------------------------------------------------------------
    patches.patch_draft_lm_head()
    V, H, num_pad = 16384 + 640, 256, 64
    rs = np.random.RandomState(3000)
    wf = rs.standard_normal((V, H)).astype(np.float32) * 0.05
    wf[7] = 0.0                        # all-zero row: exercises the 1e-8 clamp
    wf[11, 3] = 40.0                   # one large outlier in a row
    w_bits = orc.f32_to_bf16(wf)
    lm_head = types.SimpleNamespace(weight=bits_to_bf16(w_bits), tp_size=1,
                                    shard_indices=types.SimpleNamespace(num_org_vocab_padding=num_pad,
                                                                        org_vocab_start_index=0))
    draft = MTP()
    draft.lm_head = lm_head
    draft.logits_processor = types.SimpleNamespace(logits_as_input=False, soft_cap=None, scale=1.0,
                                                   org_vocab_size=V - num_pad)
    spec = Spec()
    spec.draft = draft
    Spec.load_draft_model(spec, None, None)
    w_t, scale, npad, cfg = draft._qf_head_i8
    w8 = w_t.t().contiguous().numpy()
    rows = np.r_[0:32, 16368:16400, V - 32:V]      # both sides of the 16384-row quantizer block edge
    arrays["head_w8_rows"] = w8[rows]
    arrays["head_w8_row_index"] = rows
    arrays["head_scale"] = scale.numpy()
    head = {"V": V, "H": H, "num_pad": int(npad), "cfg": cfg, "weight_seed": 3000,
            "weight_sha256": sha(w_bits), "w8_sha256": sha(w8), "cases": []}
    for k, M in enumerate((1, 3, 4)):
        seed = 3100 + k
        hs_bits = orc.f32_to_bf16(np.random.RandomState(seed).standard_normal((M, H)).astype(np.float32))
        hs = bits_to_bf16(hs_bits)
        logits = MTP.compute_logits(draft, hs)
        top = MTP.get_top_tokens(draft, hs)
        arrays[f"head{k}_logits"] = bf16_to_bits(logits)
        arrays[f"head{k}_top"] = top.numpy().astype(np.int64)
        head["cases"].append({"case": k, "M": M, "seed": seed, "logits_shape": list(logits.shape)})
        print(f"head case {k}: M={M} top={top.tolist()}", flush=True)
    meta["head"] = head

    out = Path(args.out)
    np.savez_compressed(out / "reference_outputs.npz", **arrays)
    (out / "reference_outputs.json").write_text(json.dumps(meta, indent=1, default=list) + "\n")
    print("wrote", out / "reference_outputs.npz")


if __name__ == "__main__":
    main()
