"""Generate tests/golden/*.npz from the REFERENCE's own CPU code.

Runs in the development container, where oracle/Makefile has compiled the
reference's src/quant.cc (and the files it needs) into
oracle/_ref/libref_scalar.so.  The fixtures it writes are the reference's
outputs on seeded inputs, committed so the CPU tests can pin the oracle on
machines without the reference checkout:

    make -C oracle ref && python tests/golden/make_golden.py

Cases
  * q8_0 / q4_0: quantizeToQ80/Q40 -> blocks, dequantizeFromQ80/Q40 -> w,
    linearQ80/Q40 on 1-D and 2-D x (quant.cc:130-302, 401-475, 630-644).
    Shapes include partial last blocks (cols 100, 33, 1) and 3-block rows.
  * q4_1 (no reference quantizer): seeded random blocks with finite d, m;
    dequantizeFromQ41 and linearQ41 (quant.cc:350-392, 646-650).
  * The fillLinear inputs of the reference's GPU tests
    (tests/test_cuda.cc:66-77, 679-743, makeQ41Blocks :115-131).
  * swiGlu (src/ops.cc:111-145) on gate values spanning -100..100 (exp
    overflow and underflow included) and on the outputs of two q4_0 linears
    sharing one x (the fused gate/up case).
The inputs come from the seeded generator of mini-llama_b200/synth.py.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
from oracle.oracle import Reference  # noqa: E402

_spec = importlib.util.spec_from_file_location("mlq_synth", ROOT / "mini-llama_b200" / "synth.py")
synth = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(synth)

SHAPES = [(4, 32), (7, 100), (3, 96), (8, 1024), (5, 1), (2, 33), (6, 64)]


def fill_linear(n: int, scale: float, offset: float) -> np.ndarray:
    # tests/test_cuda.cc:66-77: t[i] = offset + scale * i (fp32 arithmetic)
    i = np.arange(n, dtype=np.float32)
    return (np.float32(offset) + np.float32(scale) * i).astype(np.float32)


def q41_test_blocks(out_f: int, in_f: int) -> np.ndarray:
    # tests/test_cuda.cc:115-131: d = fp16(0.5), m = 0, qs[i] = ((3i+1)&15) | ((5i+2)&15)<<4
    nb = out_f * ((in_f + 31) // 32)
    blk = np.zeros((nb, 20), dtype=np.uint8)
    blk[:, 0], blk[:, 1] = 0x00, 0x38
    for i in range(16):
        blk[:, 4 + i] = ((i * 3 + 1) & 0x0F) | (((i * 5 + 2) & 0x0F) << 4)
    return blk.reshape(-1)


def random_q41_blocks(rows: int, cols: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    nb = rows * ((cols + 31) // 32)
    blk = rng.integers(0, 256, size=(nb, 20), dtype=np.uint8)
    for off in (0, 2):  # finite d and m: exponent field < 31
        h = (rng.integers(0x0400, 0x6000, size=nb) | (rng.integers(0, 2, size=nb) << 15)).astype(np.uint16)
        blk[:, off] = h & 0xFF
        blk[:, off + 1] = h >> 8
    return blk.reshape(-1)


def main() -> None:
    ref = Reference("scalar")
    ref.set_threads(1)
    out = {}
    for fmt in ("q8_0", "q4_0"):
        for si, (rows, cols) in enumerate(SHAPES):
            key = f"{fmt}_{rows}x{cols}"
            w = synth.normal((rows, cols), seed=1000 + si, std=0.02)
            blocks = ref.quantize(fmt, w)
            out[f"{key}_w"] = w
            out[f"{key}_blocks"] = blocks
            out[f"{key}_deq"] = ref.dequantize(fmt, blocks, rows, cols)
            for xr in (0, 3):
                x = synth.normal((cols,) if xr == 0 else (xr, cols), seed=2000 + si + xr, std=1.0)
                out[f"{key}_x{xr}"] = x
                out[f"{key}_y{xr}"] = ref.linear(fmt, x, blocks, rows)
    for si, (rows, cols) in enumerate(SHAPES):
        key = f"q4_1_{rows}x{cols}"
        blocks = random_q41_blocks(rows, cols, 3000 + si)
        out[f"{key}_blocks"] = blocks
        out[f"{key}_deq"] = ref.dequantize("q4_1", blocks, rows, cols)
        for xr in (0, 3):
            x = synth.normal((cols,) if xr == 0 else (xr, cols), seed=4000 + si + xr, std=1.0)
            out[f"{key}_x{xr}"] = x
            out[f"{key}_y{xr}"] = ref.linear("q4_1", x, blocks, rows)
    # the reference GPU tests' own inputs (tests/test_cuda.cc:679-743)
    wt = fill_linear(4 * 32, 0.05, -1.0).reshape(4, 32)
    xt = fill_linear(32, 0.1, -0.4)
    x2 = fill_linear(64, 0.07, -0.3).reshape(2, 32)
    out["tc_w"], out["tc_x"], out["tc_x2"] = wt, xt, x2
    out["tc_bias"] = fill_linear(4, 0.2, -0.1)
    for fmt in ("q8_0", "q4_0"):
        b = ref.quantize(fmt, wt)
        out[f"tc_{fmt}_blocks"] = b
        out[f"tc_{fmt}_y"] = ref.linear(fmt, xt, b, 4)
        out[f"tc_{fmt}_y2"] = ref.linear(fmt, x2, b, 4)
    b41 = q41_test_blocks(4, 32)
    out["tc_q4_1_blocks"] = b41
    out["tc_q4_1_y"] = ref.linear("q4_1", xt, b41, 4)
    # swiGlu: elementwise edge values, then a gate/up pair of q4_0 linears
    g = np.concatenate([np.linspace(-100.0, 100.0, 101, dtype=np.float32),
                        synth.normal((155,), seed=5000, std=4.0)]).astype(np.float32)
    u = synth.normal((256,), seed=5001, std=1.0)
    out["swiglu_gate"], out["swiglu_up"] = g, u
    out["swiglu_h"] = ref.swiglu(g, u)
    wg = synth.normal((48, 256), seed=5002, std=0.02)
    wu = synth.normal((48, 256), seed=5003, std=0.02)
    xs = synth.normal((3, 256), seed=5004, std=1.0)
    bg, bu = ref.quantize("q4_0", wg), ref.quantize("q4_0", wu)
    yg, yu = ref.linear("q4_0", xs, bg, 48), ref.linear("q4_0", xs, bu, 48)
    out["ffn_gate_blocks"], out["ffn_up_blocks"], out["ffn_x"] = bg, bu, xs
    out["ffn_h"] = np.stack([ref.swiglu(yg[r], yu[r]) for r in range(3)])
    np.savez_compressed(HERE / "reference_quant.npz", **out)
    print(f"wrote {len(out)} arrays to {HERE / 'reference_quant.npz'}")


if __name__ == "__main__":
    main()
