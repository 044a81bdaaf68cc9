"""Records the accuracy of the reference's own CUDA path on every parity case.

Run on a GPU box (writes ``tests/golden/fla_accuracy.json``)::

    python tests/golden/make_fla_accuracy.py [--only CASE ...]

For each case of ``cases.ALL_CASES`` the inputs are rounded to bf16, the float64
oracle is run on them, and so is the reference's CUDA path: a bf16 conv1d+SiLU
(``ml/runtime/model/attention.py:32-60`` under autocast) followed by
flash-linear-attention's Triton ``chunk_kda`` (``attention.py:349-365``;
``FLA_DISABLE_BACKEND_DISPATCH=1`` so the default Triton kernels run).  The
per-tensor errors (``viol``: max |x - ref| / (atol*max(1, rms) + rtol |ref|)
with rtol 2e-2 / atol 2e-3, and ``rel``: relative Frobenius error) are stored;
the GPU parity tests hold the B200 kernels to "within tolerance, or no less
accurate than this reference path".  flash-linear-attention's version is
recorded alongside (Sophia pins 0.5.2; the image ships 0.5.1).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE.parent.parent))

os.environ.setdefault("FLA_DISABLE_BACKEND_DISPATCH", "1")

from cases import ALL_CASES, make_case_inputs  # noqa: E402
from fla_runner import run_fla  # noqa: E402
from kda_cuda_runner import compare, round_inputs_bf16  # noqa: E402
from oracle_runner import run_oracle  # noqa: E402


def parity_cases() -> dict:
    """Every case the GPU parity tests compare with a recorded baseline: the
    fixture and random cases plus one configuration-4 packed window."""
    from cases import LONG_CASES, cfg4_case
    c4 = cfg4_case(0, H=4)
    return {**ALL_CASES, c4.name: c4, **LONG_CASES}


def main() -> None:
    import argparse

    import fla
    import numpy as np
    import torch
    from cases import CASES
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*", default=None,
                    help="recompute these case names and keep the other recorded entries")
    a = ap.parse_args()
    path = HERE / "fla_accuracy.json"
    if a.only is not None and path.exists():
        with open(path) as f:
            out = json.load(f)
    else:
        out = {"fla_version": getattr(fla, "__version__", "unknown"), "cases": {}, "golden": {}}
    for name, case in parity_cases().items():
        if a.only is not None and name not in a.only:
            continue
        inp = round_inputs_bf16(make_case_inputs(case))
        ref = run_oracle(case, inputs=inp)
        rep = compare(run_fla(case, inputs=inp), ref)
        out["cases"][name] = {k: {"viol": v[0], "rel": v[1]} for k, v in rep.items()}
        print(name, flush=True)
    # against the reference's own float32 outputs on the unrounded inputs
    for name, case in CASES.items():
        if a.only is not None and name not in a.only:
            continue
        gold = np.load(HERE / f"{name}.npz")
        ref = {k: torch.from_numpy(gold[k]) for k in gold.files if k != "input_sums"}
        rep = compare(run_fla(case), ref)
        out["golden"][name] = {k: {"viol": v[0], "rel": v[1]} for k, v in rep.items()}
        print("golden", name, flush=True)
    with open(path, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
