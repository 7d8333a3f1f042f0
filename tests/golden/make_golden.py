"""Generate the committed golden fixtures from the reference itself.

Run in a container where the reference checkout is mounted (it is absent on GPU
hosts): ``python tests/golden/make_golden.py --ref <reference checkout>``.

Sources of truth, all from the reference:
  * its numpy specification of the decoder ops - ``rms_norm``, ``rope_neox`` and
    ``silu`` from tools/verify_xfmr.py:32-80 (the MLP is ``silu(gate) * up``,
    tools/verify_xfmr.py:181) and ``snake_beta`` from tools/verify_vocoder.py:152-157.
    Those scripts load model weights at import, so only the named function
    definitions are taken out of their syntax trees and executed.
  * its compiled ``voc_snake_beta`` (src/tts_vocoder_ops.c:279-305), built by
    oracle/Makefile into oracle/_ref/ in the scalar and the shipped AVX2 form.
  * the BF16->F32 widening of src/tts_native.c:35-40, whose known answers on
    special bit patterns are written out by hand (the function is static in a
    file that needs the absent qwen-asr headers, so it cannot be linked).

Inputs are seeded, small, and stored beside the outputs in .npz files.
"""
from __future__ import annotations

import argparse
import ast
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))


def extract_functions(path: str, names: list[str]) -> dict:
    """Execute only the named top-level function definitions of a script."""
    with open(path) as f:
        tree = ast.parse(f.read(), filename=path)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in keep}
    if missing:
        raise RuntimeError(f"{path}: functions not found: {sorted(missing)}")
    mod = ast.Module(body=keep, type_ignores=[])
    ns: dict = {"np": np}
    exec(compile(mod, path, "exec"), ns)
    return {n: ns[n] for n in names}


def main() -> None:
    ap = argparse.ArgumentParser()
    beside = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "..", "reference")
    ap.add_argument("--ref", default=os.environ.get("LAI_REFERENCE", os.path.normpath(beside)),
                    help="the reference checkout (default: $LAI_REFERENCE, else a reference/ "
                         "directory beside this repository)")
    args = ap.parse_args()
    ref = args.ref
    xf = extract_functions(os.path.join(ref, "tools", "verify_xfmr.py"),
                           ["rms_norm", "rope_neox", "silu"])
    vc = extract_functions(os.path.join(ref, "tools", "verify_vocoder.py"), ["snake_beta"])

    import oracle  # noqa: E402  (builds oracle/_ref from the reference source if needed)
    oracle.build()

    rng = np.random.default_rng(20261201)
    out = {}

    # RMSNorm: decoder eps 1e-6 (src/tts_native.h:42) at D=1024 and 2048, vocoder
    # eps 1e-5 (src/tts_vocoder.h:42) at D=512, plus a ragged width.
    for tag, (seq, dim, eps) in {"d1024": (16, 1024, 1e-6), "d2048": (8, 2048, 1e-6),
                                 "d512": (16, 512, 1e-5), "d200": (5, 200, 1e-6)}.items():
        x = rng.standard_normal((seq, dim), dtype=np.float32)
        w = (1.0 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
        y = xf["rms_norm"](x, w, eps=eps).astype(np.float32)
        out[f"rmsnorm_{tag}"] = dict(x=x, w=w, eps=np.float32(eps), y=y)

    # NeoX RoPE over positions 0..T-1 (the prefill use), theta 1e6 hd 128
    # (src/tts_native.h:41) and theta 1e4 hd 64 (vocoder, src/tts_vocoder.h:39-41).
    for tag, (T, heads, hd, theta) in {"hd128": (24, 4, 128, 1e6), "hd64": (24, 16, 64, 1e4)}.items():
        x = rng.standard_normal((T, heads * hd), dtype=np.float32)
        y = xf["rope_neox"](x.copy(), T, heads, hd, theta=theta).astype(np.float32)
        out[f"rope_{tag}"] = dict(x=x, theta=np.float32(theta), heads=np.int32(heads),
                                  hd=np.int32(hd), y=y)

    # SwiGLU: gate/up rows interleaved as the fused weight makes them
    # (src/tts_native.c:149-161); reference math silu(gate) * up.
    seq, inter = 6, 384
    gate = (2.0 * rng.standard_normal((seq, inter))).astype(np.float32)
    up = rng.standard_normal((seq, inter), dtype=np.float32)
    gate_up = np.empty((seq, 2 * inter), np.float32)
    gate_up[:, 0::2] = gate
    gate_up[:, 1::2] = up
    out["swiglu"] = dict(gate_up=gate_up, inter=np.int32(inter),
                         y=(xf["silu"](gate) * up).astype(np.float32))
    s = (4.0 * rng.standard_normal(4096)).astype(np.float32)
    out["silu"] = dict(x=s, y=xf["silu"](s).astype(np.float32))

    # SnakeBeta: numpy spec and the reference's compiled function (both builds).
    C, T = 12, 257
    x = rng.standard_normal((C, T), dtype=np.float32)
    alpha = (0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    ea = np.exp(alpha).astype(np.float32)
    ieb = (1.0 / np.exp(beta)).astype(np.float32)
    y_np = vc["snake_beta"](x, alpha, beta).astype(np.float32)
    y_ref = oracle.ref_snake_beta(x, ea, ieb, "scalar")
    y_avx = oracle.ref_snake_beta(x, ea, ieb, "avx2")
    out["snake"] = dict(x=x, alpha=alpha, beta=beta, ea=ea, ieb=ieb, y_numpy=y_np,
                        y_ref_scalar=y_ref, y_ref_avx2=y_avx)

    # BF16 -> F32 widening known answers (src/tts_native.c:35-40: bits << 16).
    pats = np.array([0x0000, 0x8000, 0x0001, 0x807F, 0x3F80, 0xBF80, 0x7F7F, 0x7F80, 0xFF80,
                     0x7FC0, 0xFFC1, 0x7F81, 0x4049, 0xC2F7, 0x0080, 0x3C00], np.uint16)
    widened = (pats.astype(np.uint32) << 16).astype(np.uint32)
    out["bf16_widen"] = dict(bf16=pats, f32_bits=widened)

    for name, d in out.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
    print(f"wrote {len(out)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
