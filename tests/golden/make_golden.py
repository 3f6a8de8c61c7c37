"""Generate the golden fixtures in this directory from the reference's own CUDA kernels.

Run on a B200 after ``python oracle/build_ref.py`` (which compiles the unmodified
reference ``attention.cu`` per compile-time variant into ``oracle/_ref``):

    python tests/golden/make_golden.py [out_dir]

For each case the seeded fp16 inputs (``morphottention_b200.configs.make_inputs``) are run
through the reference forward and backward (grad_out = ones, i.e. ``out.sum()``); the
outputs are stored as ``<case>.npz`` (inputs are not stored: they are regenerated from the
seed).  ``tests/test_golden_cpu.py`` checks the CPU oracle against these files.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from morphottention_b200.configs import CONFIGS, MorphoConfig, make_inputs  # noqa: E402
from oracle import refkernel  # noqa: E402

CASES = {
    # name: (config, random_gates)
    "c1_readme_gates1": (CONFIGS["c1"], False),
    "c1_readme_gatesR": (CONFIGS["c1"], True),
    "narrow_causal_m16": (MorphoConfig("narrow_causal_m16", 1, 256, 128, 2, 16, 1.0, True, 21), True),
    "narrow_m32_n197": (MorphoConfig("narrow_m32_n197", 1, 197, 128, 2, 32, 0.5, False, 22), True),
}


def main(out_dir: str) -> None:
    os.makedirs(out_dir, exist_ok=True)
    meta = {}
    for name, (cfg, gates) in CASES.items():
        inp = make_inputs(cfg, device="cuda", random_gates=gates)
        out, lse = refkernel.forward(cfg, inp)
        grads = refkernel.backward(cfg, inp, out, lse, torch.ones_like(out))
        torch.cuda.synchronize()
        arrays = {"out": out, "lse": lse, **grads}
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"),
                            **{k: v.detach().cpu().numpy() for k, v in arrays.items()})
        meta[name] = {"config": cfg.__dict__, "random_gates": gates, "grad_out": "ones",
                      "reference_variant": refkernel.VARIANT_OF[(cfg.cube_m, cfg.head_dim, cfg.causal)],
                      "device": torch.cuda.get_device_name()}
        print(name, {k: float(v.float().abs().mean()) for k, v in arrays.items()})
    with open(os.path.join(out_dir, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
