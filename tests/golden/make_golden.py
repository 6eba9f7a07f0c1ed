"""Generate golden forward vectors from the reference's own CPU implementation.

Runs ``cron_root_attention.cpu_reference.cra_cpu_fast`` (the function the
reference dispatches to for CPU tensors, core.py:3794-3796) on small seeded
inputs and stores inputs + outputs under ``tests/golden/``.  The reference
package must be importable (pass its checkout root as argv[1]); it is only
needed to regenerate the fixtures, never at test time.

The reference's CPU path uses W = isqrt(S) (cpu_reference.py:233) while its
GPU path uses W = ceil(sqrt(S)) (core.py:3479).  For non-square S the module's
``math`` binding is swapped for a namespace whose ``isqrt`` returns
ceil(sqrt(n)), so the stored outputs follow the GPU semantics without editing
the reference.  The GPU path also skips the relay for S <= 2048
(core.py:3507); those cases call ``cra_cpu_fast(..., use_relay=False)``.

Inputs are drawn in fp32 from ``torch.Generator().manual_seed(seed)`` and
rounded to the case's storage dtype; the reference runs on the fp32 upcast of
the rounded values.

Usage: python tests/golden/make_golden.py <reference_checkout_root>
"""
import math
import os
import sys
import types

import numpy as np
import torch

CASES = [
    # name, B, H, S, D, dtype, seed, sigma
    ("s300_d64_f16", 1, 2, 300, 64, torch.float16, 10, 1.0),      # relay off, non-square
    ("s2304_d64_f16", 1, 1, 2304, 64, torch.float16, 11, 1.0),    # 48^2, relay on
    ("s3001_d64_bf16", 1, 1, 3001, 64, torch.bfloat16, 12, 1.0),  # non-square: ceil W = 55
    ("s2116_d128_bf16", 1, 1, 2116, 128, torch.bfloat16, 13, 1.0),  # 46^2, relay on
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import cron_root_attention.cpu_reference as cr  # noqa: E402

    shim = types.SimpleNamespace(**{n: getattr(math, n) for n in dir(math) if not n.startswith("_")})
    shim.isqrt = lambda n: int(math.ceil(math.sqrt(n)))
    cr.math = shim
    out_dir = os.path.dirname(os.path.abspath(__file__))
    for name, B, H, S, D, dt, seed, sigma in CASES:
        g = torch.Generator().manual_seed(seed)
        q = (torch.randn(B, H, S, D, generator=g) * sigma).to(dt)
        k = (torch.randn(B, H, S, D, generator=g) * sigma).to(dt)
        v = (torch.randn(B, H, S, D, generator=g) * sigma).to(dt)
        use_relay = S > 2048
        with torch.no_grad():
            o = cr.cra_cpu_fast(q.float(), k.float(), v.float(), use_relay=use_relay)
        st = np.float16 if dt == torch.float16 else np.uint16  # bf16 stored as raw bits
        def raw(t):
            return t.contiguous().view(torch.int16).numpy().view(np.uint16) if dt == torch.bfloat16 \
                else t.numpy().astype(st)
        np.savez_compressed(
            os.path.join(out_dir, name + ".npz"),
            q=raw(q), k=raw(k), v=raw(v), out=o.numpy().astype(np.float32),
            meta=np.array([B, H, S, D, int(use_relay), seed], dtype=np.int64),
            dtype=np.array("bf16" if dt == torch.bfloat16 else "f16"),
        )
        print(name, "written", tuple(o.shape))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "..")
