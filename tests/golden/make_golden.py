"""Regenerate tests/golden/ from the reference's own CPU selection restatement.

Runs only where the reference checkout is present (its location comes from
REFERENCE_ROOT, with the build container's checkout as the default).  It imports verify_selection_flow.py from the
reference, walks its 47 fixtures with their layouts (fixtures() :168-199,
backing_and_view() :202-213), evaluates its ``reference()`` (:27-47) and
stores inputs and all 8 trace outputs as raw bits, plus the reference's
score_key / float_bits over all 65,536 fp16 patterns (:72-93).

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def bits(t):
    import torch
    t = t.contiguous()
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


def main() -> None:
    root = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
    sys.path.insert(0, str(root))
    os.environ["TORCH_DEVICE_BACKEND_AUTOLOAD"] = "0"
    import torch
    import verify_selection_flow as ref  # the reference's CPU-only checker

    torch.set_num_threads(1)
    torch.manual_seed(149)
    ref.cpu_algorithm_checks()
    halves = np.arange(65536, dtype=np.uint32)
    np.savez_compressed(HERE / "selection_keys.npz",
                        score_key=np.array([ref.score_key(int(h)) for h in halves], np.uint32),
                        float_bits=np.array([ref.float_bits(int(h)) for h in halves], np.uint32))
    out_dir = HERE / "selection"
    out_dir.mkdir(exist_ok=True)
    index = []
    with torch.inference_mode():
        for name, x, max_det, agnostic, layout, unique in ref.fixtures():
            base, view = ref.backing_and_view(x, layout)
            x = view(base)
            expected = ref.reference(x, max_det, agnostic)
            arrays = {"decoded": bits(x)}
            for key in ref.TRACE_NAMES:
                arrays[key] = bits(expected[key])
            np.savez_compressed(out_dir / f"{name}.npz", **arrays)
            index.append(dict(name=name, max_det=int(max_det), agnostic=bool(agnostic), layout=layout,
                              shape=list(x.shape), stride=list(x.stride()), unique=bool(unique)))
    (HERE / "selection_index.json").write_text(json.dumps(index, indent=1) + "\n")
    print(f"wrote {len(index)} selection fixtures")


if __name__ == "__main__":
    main()
