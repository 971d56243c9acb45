"""Records golden vectors of the B200's stochastic-rounding conversions (run on a B200).

The reference's stochastic conversions are the hardware cvt.rs instructions
(src/data_types/narrow.rs:217-229, bfloat16.rs:456-462, float16.rs:589-595), so the device's own
outputs are the golden answers. For each of the 18 forms (five x4 formats with and without
.relu; bf16 and f16 with every .relu/.satfinite combination) the script converts 512 groups of
seeded inputs through the library's element-wise entry points and stores the f32 input bit
patterns, the rbits words and the codes:

    python tests/golden/make_cvt_rs_vectors.py --out tests/golden/cvt_rs_vectors.json

Inputs: random signs, exponents across each format's range (its subnormals and some overflow
included), mantissas either random or with only the top bits set, plus zeros, infinities, NaNs,
f32 subnormals; rbits: random words, 0, all ones and single bits.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "ptx-std_b200")]

# name: (elements per group, lowest and highest unbiased exponent drawn)
FORMS = {
    "e4m3": (4, -12, 10), "e5m2": (4, -19, 17), "e2m3": (4, -5, 4), "e3m2": (4, -7, 6),
    "e2m1": (4, -3, 4), "bf16": (2, -136, 128), "f16": (2, -27, 17),
}
GROUPS = 512


def inputs(name: str, seed: int):
    per, lo, hi = FORMS[name]
    rng = np.random.default_rng(seed)
    n = GROUPS * per
    e = rng.integers(lo, hi + 1, n)
    m = rng.integers(0, 1 << 23, n, dtype=np.int64)
    sparse = rng.random(n) < 0.3
    m[sparse] &= ~((1 << rng.integers(8, 23, int(sparse.sum()))) - 1)
    bits = ((rng.integers(0, 2, n) << 31) | (np.clip(e + 127, 0, 255) << 23) | m).astype(np.uint32)
    sp = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00001, 0x00000001,
                   0x807FFFFF], dtype=np.uint32)
    bits[: sp.size] = sp
    rb = rng.integers(0, 1 << 32, GROUPS, dtype=np.uint64).astype(np.uint32)
    rb[:34] = [0, 0xFFFFFFFF] + [1 << b for b in range(32)]
    return bits, rb


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "cvt_rs_vectors.json"))
    a = ap.parse_args()
    import torch

    import ptxstd.data_types as dt

    out = {"device": torch.cuda.get_device_name(), "forms": {}}
    for i, (name, (per, _, _)) in enumerate(FORMS.items()):
        bits, rb = inputs(name, 9000 + i)
        x = torch.from_numpy(bits.view(np.float32)).cuda()
        r = torch.from_numpy(rb.view(np.int32)).cuda()
        variants = ([(relu, True) for relu in (False, True)] if per == 4 else
                    [(relu, sat) for sat in (False, True) for relu in (False, True)])
        for relu, sat in variants:
            if per == 4:
                codes = dt.from_f32_stochastic(name, x, r, relu=relu).cpu().numpy()
                codes = codes.view(np.uint8)
            elif name == "bf16":
                codes = dt.bf16_from_f32_stochastic(x, r, relu, sat).cpu().numpy().view(np.uint16)
            else:
                codes = dt.f16_from_f32_stochastic(x, r, relu, sat).cpu().numpy().view(np.uint16)
            torch.cuda.synchronize()
            key = name + ("_relu" if relu else "") + ("_sat" if per == 2 and sat else "")
            out["forms"][key] = {"x": [f"{v:08x}" for v in bits], "rbits": [f"{v:08x}" for v in rb],
                                 "codes": codes.tobytes().hex()}
            print(key, flush=True)
    with open(a.out, "w") as f:
        json.dump(out, f, indent=0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
