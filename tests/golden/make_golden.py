"""Generate the golden vectors by running the reference's own PyTorch CPU path.

Run once in a container where the reference project is mounted:

    python tests/golden/make_golden.py <reference project directory>

(or with the directory in ``BS_REFERENCE_DIR``).

It imports the reference module ``kernel_sm121`` and calls ``act_quant``,
``fp4_act_quant``, ``fp8_gemm`` and ``fp4_gemm`` on CPU tensors (the branch
taken when ``a.is_cuda`` is false), on seeded numpy inputs, and writes
``golden.npz`` beside this file.  Large operands are not stored: the file
keeps the generator seed and a sha256 of the bytes instead, and the tests
regenerate them with ``tests/golden/cases.py``.

The MoE case composes the reference ops the same way ``oracle.moe_layer``
does (the reference's own MoE caller lives in an external model file that is
not part of the reference project).
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def t_bf16(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def t_u8(u8, dtype):
    return torch.from_numpy(np.ascontiguousarray(u8)).view(dtype)


def np_bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e8m0fnu, torch.uint8):
        return t.contiguous().view(torch.uint8).numpy()
    return t.contiguous().numpy()


def main(ref_dir: str) -> None:
    sys.path.insert(0, ref_dir)
    import kernel_sm121 as ks  # the reference module

    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    out = {}

    # --- act_quant -------------------------------------------------------
    for name, (x, xdt) in cases.act_quant_inputs().items():
        xt = t_bf16(x) if xdt == "bf16" else torch.from_numpy(x)
        out[f"aq/{name}/x"] = x
        for fmt in (None, "ue8m0"):
            for sdt_name, sdt in (("f32", torch.float32), ("e8m0", torch.float8_e8m0fnu)):
                y, s = ks.act_quant(xt.clone(), 128, fmt, sdt, False)
                key = f"aq/{name}/{fmt}/{sdt_name}"
                out[key + "/y"] = np_bits(y)
                out[key + "/s"] = np_bits(s)
            r = ks.act_quant(xt.clone(), 128, fmt, torch.float32, True)
            out[f"aq/{name}/{fmt}/inplace"] = np_bits(r)

    # --- fp4_act_quant ---------------------------------------------------
    for name, (x, xdt) in cases.fp4_act_quant_inputs().items():
        xt = t_bf16(x) if xdt == "bf16" else torch.from_numpy(x)
        out[f"f4q/{name}/x"] = x
        r = ks.fp4_act_quant(xt.clone(), 32, True)
        out[f"f4q/{name}/out"] = np_bits(r)

    # --- fp8_gemm --------------------------------------------------------
    for name, c in cases.fp8_gemm_cases().items():
        a, a_s, b, b_s = c["a"], c["a_s"], c["b"], c["b_s"]
        at = t_u8(a, torch.float8_e4m3fn)
        bt = t_u8(b, torch.float8_e4m3fn)
        ast = torch.from_numpy(a_s) if c["as_dt"] == "f32" else t_u8(a_s, torch.float8_e8m0fnu)
        bst = torch.from_numpy(b_s) if c["bs_dt"] == "f32" else t_u8(b_s, torch.float8_e8m0fnu)
        o = np_bits(ks.fp8_gemm(at, ast, bt, bst))
        # large outputs keep every 256th row only (rows are independent)
        out[f"g8/{name}/out"] = o[::256] if o.shape[0] > 1024 else o
        for k in ("a", "a_s", "b", "b_s"):
            out[f"g8/{name}/sha_{k}"] = np.array(sha(c[k]))

    # --- fp4_gemm --------------------------------------------------------
    for name, c in cases.fp4_gemm_cases().items():
        a, a_s, b, b_s = c["a"], c["a_s"], c["b"], c["b_s"]
        at = t_u8(a, torch.float8_e4m3fn)
        bt = t_u8(b, torch.float4_e2m1fn_x2)
        ast = torch.from_numpy(a_s) if c["as_dt"] == "f32" else t_u8(a_s, torch.float8_e8m0fnu)
        bst = t_u8(b_s, torch.float8_e8m0fnu)
        o = ks.fp4_gemm(at, ast, bt, bst)
        out[f"g4/{name}/out"] = np_bits(o)
        for k in ("a", "a_s", "b", "b_s"):
            out[f"g4/{name}/sha_{k}"] = np.array(sha(c[k]))

    # --- composed MoE ----------------------------------------------------
    m = cases.moe_case_small()
    x = t_bf16(m["x"])
    idx, w = m["idx"], m["w"]
    E, twoI, _ = m["w13"].shape
    inter = twoI // 2
    acc = torch.zeros(x.shape, dtype=torch.float32)
    for e in range(E):
        tok, slot = np.nonzero(idx == e)
        if tok.size == 0:
            continue
        h, hs = ks.act_quant(x[torch.from_numpy(tok)], 128, "ue8m0", torch.float32)
        gu = ks.fp4_gemm(h, hs, t_u8(m["w13"][e], torch.float4_e2m1fn_x2),
                         t_u8(m["w13_s"][e], torch.float8_e8m0fnu)).float()
        g, u = gu[:, :inter], gu[:, inter:]
        z = torch.nn.functional.silu(g) * u
        q, qs = ks.act_quant(z, 128, "ue8m0", torch.float32)
        y = ks.fp4_gemm(q, qs, t_u8(m["w2"][e], torch.float4_e2m1fn_x2),
                        t_u8(m["w2_s"][e], torch.float8_e8m0fnu)).float()
        ww = torch.from_numpy(w[tok, slot])[:, None]
        acc.index_add_(0, torch.from_numpy(tok), ww * y)
    out["moe/small/out"] = np_bits(acc.to(torch.bfloat16))
    out["moe/small/sha_w13"] = np.array(sha(m["w13"]))

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("BS_REFERENCE_DIR", "")
    if not ref:
        sys.exit("usage: make_golden.py <reference project directory> (or set BS_REFERENCE_DIR)")
    main(ref)
