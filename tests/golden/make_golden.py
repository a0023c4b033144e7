"""Generate the golden fixtures that pin the CPU oracle to the reference.

Two steps, two machines:

``python tests/golden/make_golden.py inputs PATH/TO/REFERENCE_IMPL.md``  (needs the reference tree)
    The listing file is the argument, or the NVFP4_REFERENCE_IMPL environment variable.
    Executes the reference harness's own Python listings from
    ``REFERENCE_IMPL.md`` (``to_blocked``, ``create_reordered_scale_factor_tensor``,
    ``_create_fp4_tensors``, ``generate_input``) on the CPU -- the only change is
    that their hard-coded ``"cuda"`` device becomes ``"cpu"`` -- and stores, per
    case, the generated operands, plain scales, the reference's reordered scale
    storage and the reference's ``to_blocked`` output in ``golden_inputs.npz``.
    A few cases use the benchmark distribution (all 16 e2m1 codes, scales
    2^U{-4..3}) drawn with numpy instead.

``python tests/golden/make_golden.py outputs [out.npz]``  (a B200)
    Runs the reference's arithmetic -- ``torch._scaled_mm`` on the reference's own
    ``to_blocked`` bytes with ``out_dtype=float16``, as ``ref_kernel`` does
    (REFERENCE_IMPL.md:71-78); gated cases add ``silu(t1.float()) * t2.float()``
    as submission.py:884 does -- and stores the fp16 outputs (plus fp32 products
    for overflow analysis) in ``golden_outputs.npz``.
"""
from __future__ import annotations

import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
INPUTS = os.path.join(HERE, "golden_inputs.npz")
OUTPUTS = os.path.join(HERE, "golden_outputs.npz")
REFERENCE_IMPL = os.environ.get("NVFP4_REFERENCE_IMPL")

# (name, generator, m, n, k, seed, extra)
CASES = [
    ("ref_g2", "reference", (80, 200), (256, 256), (512, 512), 1111, {}),
    ("ref_cfg1_shape", "reference", (128,), (256,), (512,), 2222, {}),
    ("ref_g3_ragged", "reference", (40, 128, 257), (384, 128, 640), (256, 1024, 768), 3333, {}),
    ("all16_cfg1", "all16", (128,), (256,), (512,), 4444, {}),
    ("all16_g2_alpha", "all16", (64, 300), (256, 256), (1024, 1024), 5555,
     {"alpha": (0.75, 1.5)}),
    ("ref_gated", "reference", (96,), (256,), (512,), 6666, {"gated": True}),
    ("all16_gated", "all16", (200,), (384,), (768,), 7777, {"gated": True}),
]


def _load_reference_namespace():
    import torch

    if not REFERENCE_IMPL:
        sys.exit("the reference's REFERENCE_IMPL.md is needed: pass its path after `inputs` "
                 "or set NVFP4_REFERENCE_IMPL")
    src = open(REFERENCE_IMPL).read()
    blocks = re.findall(r"```python\n(.*?)```", src, re.S)
    wanted = ("sf_vec_size", "def to_blocked", "def create_reordered_scale_factor_tensor",
              "def _create_fp4_tensors")
    code = "\n".join(b for b in blocks if any(w in b for w in wanted))
    code = (code.replace('device="cuda"', 'device="cpu"').replace("device='cuda'", "device='cpu'")
            .replace(".cuda()", ".cpu()"))
    ns = {"torch": torch}
    exec(compile(code, REFERENCE_IMPL, "exec"), ns)
    return ns


def _u8(t):
    import torch

    return t.contiguous().view(torch.uint8).numpy().copy()


def make_inputs() -> None:
    import torch

    ns = _load_reference_namespace()
    out = {}
    for name, kind, ms, ns_, ks, seed, extra in CASES:
        gated = extra.get("gated", False)
        out[f"{name}/meta"] = np.array([len(ms), int(gated)], dtype=np.int64)
        out[f"{name}/sizes"] = np.array([(m, n, k) for m, n, k in zip(ms, ns_, ks)], dtype=np.int64)
        out[f"{name}/alpha"] = np.array(extra.get("alpha", (1.0,) * len(ms)), dtype=np.float32)
        rng = np.random.default_rng(seed)
        torch.manual_seed(seed)
        for g, (m, n, k) in enumerate(zip(ms, ns_, ks)):
            mats = {"a": m, "b": n}
            if gated:
                mats["b2"] = n
            for key, rows in mats.items():
                if kind == "reference":
                    # _create_fp4_tensors (REFERENCE_IMPL.md:143-151), then scales as generate_input
                    q = ns["_create_fp4_tensors"](1, rows, k)[:, :, 0]
                    sf = torch.randint(1, 3, (1, rows, k // 16), dtype=torch.int8).to(
                        dtype=torch.float8_e4m3fn).permute(1, 2, 0)
                else:
                    q = torch.from_numpy(rng.integers(0, 256, (rows, k // 2), dtype=np.uint8))
                    e = rng.integers(-4, 4, (rows, k // 16))
                    sf = torch.from_numpy(((e + 7) << 3).astype(np.uint8)).view(
                        torch.float8_e4m3fn)[:, :, None]
                reordered = ns["create_reordered_scale_factor_tensor"](1, rows, k, sf)
                blocked = ns["to_blocked"](sf[:, :, 0])
                out[f"{name}/{g}/{key}"] = _u8(q)
                out[f"{name}/{g}/sf_{key}"] = _u8(sf[:, :, 0])
                out[f"{name}/{g}/blocked_{key}"] = _u8(blocked)
                out[f"{name}/{g}/reordered_{key}"] = _u8(reordered.permute(5, 2, 4, 0, 1, 3))
    np.savez_compressed(INPUTS, **out)
    print(f"wrote {INPUTS} ({os.path.getsize(INPUTS)} bytes)")


def make_outputs(path: str) -> None:
    import torch

    data = np.load(INPUTS)
    names = sorted({k.split("/")[0] for k in data.files})
    out = {}
    dev = torch.device("cuda")

    def scaled_mm(a, b, sa, sb, dtype):
        return torch._scaled_mm(
            torch.from_numpy(a).to(dev).view(torch.float4_e2m1fn_x2),
            torch.from_numpy(b).to(dev).view(torch.float4_e2m1fn_x2).t(),
            torch.from_numpy(sa).to(dev).view(torch.float8_e4m3fn),
            torch.from_numpy(sb).to(dev).view(torch.float8_e4m3fn),
            bias=None, out_dtype=dtype)

    for name in names:
        G, gated = (int(x) for x in data[f"{name}/meta"])
        alpha = data[f"{name}/alpha"]
        for g in range(G):
            a = data[f"{name}/{g}/a"]
            ba = data[f"{name}/{g}/blocked_a"]
            prods = {}
            for key in (("b", "b2") if gated else ("b",)):
                b = data[f"{name}/{g}/{key}"]
                bb = data[f"{name}/{g}/blocked_{key}"]
                f16 = scaled_mm(a, b, ba, bb, torch.float16)
                f32 = scaled_mm(a, b, ba, bb, torch.float32)
                if alpha[g] != 1.0:
                    f16 = (f32 * float(alpha[g])).to(torch.float16)
                prods[key] = (f16, f32)
                out[f"{name}/{g}/fp32_{key}"] = f32.cpu().numpy()
            if gated:
                t1, t2 = prods["b"][0], prods["b2"][0]
                res = (torch.nn.functional.silu(t1.float()) * t2.float()).to(torch.float16)
            else:
                res = prods["b"][0]
            out[f"{name}/{g}/c"] = res.cpu().numpy()
    np.savez_compressed(path, **out)
    print(f"wrote {path}")


if __name__ == "__main__":
    mode = sys.argv[1] if len(sys.argv) > 1 else ""
    if mode == "inputs":
        if len(sys.argv) > 2:
            REFERENCE_IMPL = sys.argv[2]
        make_inputs()
    elif mode == "outputs":
        make_outputs(sys.argv[2] if len(sys.argv) > 2 else OUTPUTS)
    else:
        sys.exit("usage: make_golden.py inputs | outputs [out.npz]")
