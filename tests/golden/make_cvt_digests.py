"""Records digests of the B200's own `cvt` outputs over all 2^32 f32 inputs (run on a B200).

The reference's encoders are the hardware `cvt` instructions (src/data_types/narrow.rs:156-182,
:600-617), so these digests pin the oracle to the reference's conversions on a CPU-only host:
tests/test_oracle.py recomputes the oracle's digests and compares.

For each variant (e4m3, e5m2, e2m1 as one nibble per byte, the three .relu forms, ue8m0 RZ and
RP with .satfinite, the FP6 formats e2m3 and e3m2 with and without .relu, and the
stochastic-rounding forms of ptxstd_cvt_sweep 12..29, bf16/f16 with two bytes per input), the
codes of inputs [i * 2^24, (i + 1) * 2^24) are hashed as: FNV-1a 64 of every 2^16-byte piece,
then FNV-1a 64 over those digests (little-endian).

    python tests/golden/make_cvt_digests.py --out tests/golden/cvt_sweep_digests.json
    python tests/golden/make_cvt_digests.py --variants e2m3 e3m2   # add to an existing file
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "ptx-std_b200"), os.path.join(ROOT, "oracle")]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "cvt_sweep_digests.json"))
    ap.add_argument("--variants", nargs="*", default=None,
                    help="only these variants, merged into the existing --out file")
    a = ap.parse_args()
    import torch

    import oracle as O
    import ptxstd.data_types as dt

    chunk = 1 << 24
    step = 1 << 28
    dev = torch.empty(2 * step, dtype=torch.uint8, device="cuda")
    host = torch.empty(2 * step, dtype=torch.uint8, pin_memory=True)
    out = {"chunk": chunk, "scheme": "fnv1a64 of 2^16-byte pieces, then fnv1a64 of the digests",
           "device": torch.cuda.get_device_name(), "variants": {}}
    if a.variants and os.path.exists(a.out):
        out = json.load(open(a.out))
    t0 = time.time()
    for v, name in enumerate(O.VARIANT_NAMES):
        if a.variants and name not in a.variants:
            continue
        digs = []
        w = O.sweep_width(v)
        for base in range(0, 1 << 32, step):
            dt.sweep(v, base, step, out=dev)
            host.copy_(dev)
            h = host.numpy()[: w * step]
            for k in range(step // chunk):
                digs.append(f"{O.digest_bytes(h[k * chunk * w:(k + 1) * chunk * w]):016x}")
        out["variants"][name] = digs
        print(name, digs[0], f"{time.time() - t0:.1f}s", flush=True)
    with open(a.out, "w") as f:
        json.dump(out, f, indent=0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
