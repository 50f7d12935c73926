"""Generate the golden QR fixtures from the reference itself.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path-to-fast-qr-checkout>

It imports the reference's own input generator and checker
(official/reference.py: ``generate_input``, ``check_implementation``), its
PyTorch blocked compact-WY prototype (tools/blocked_qr_reference.py:
``blocked_geqrf_reference``) and its contract implementation ``torch.geqrf``
(official/reference.py:125-127), all on CPU, and stores inputs and outputs in
``golden.npz`` plus ``golden.json`` (specs and the official checker's verdict
and message).  The GPU box never runs this script; tests read the committed
fixtures only.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (name, generate_input spec).  Small cases mirror the reference's own numeric
# tests (tests/test_qr_smoke.py:170-189: batch 3, n 8); the 20 x 32 case is the
# first public test (official/task.yml:86); the rest add odd sizes, the padded
# warp sizes (33, 64) and the first sizes of the blocked path (65, 96, 130).
SPECS = [
    ("pub_20x32", dict(batch=20, n=32, cond=1, seed=53124)),
    ("s8_dense", dict(batch=3, n=8, cond=1, seed=123, case="dense")),
    ("s8_upper", dict(batch=3, n=8, cond=1, seed=124, case="upper")),
    ("s8_diagonal", dict(batch=3, n=8, cond=1, seed=125, case="diagonal")),
    ("s8_rankdef", dict(batch=3, n=8, cond=0, seed=126, case="rankdef")),
    ("s8_nearrank", dict(batch=3, n=8, cond=0, seed=127, case="nearrank")),
    ("s8_clustered", dict(batch=3, n=8, cond=0, seed=128, case="clustered")),
    ("s8_band", dict(batch=3, n=8, cond=0, seed=129, case="band")),
    ("s8_nearcollinear", dict(batch=3, n=8, cond=0, seed=130, case="nearcollinear")),
    ("s8_rowscale", dict(batch=3, n=8, cond=0, seed=131, case="rowscale")),
    ("s8_mixed", dict(batch=3, n=8, cond=1, seed=132, case="mixed")),
    ("mixed_24", dict(batch=8, n=24, cond=2, seed=133, case="mixed")),
    ("n1", dict(batch=4, n=1, cond=0, seed=134)),
    ("n2", dict(batch=4, n=2, cond=0, seed=135)),
    ("n17", dict(batch=3, n=17, cond=1, seed=136)),
    ("n33", dict(batch=3, n=33, cond=1, seed=137)),
    ("n64_graded", dict(batch=2, n=64, cond=6, seed=138)),
    ("n65", dict(batch=2, n=65, cond=1, seed=139)),
    ("n96_rankdef", dict(batch=2, n=96, cond=0, seed=140, case="rankdef")),
    ("n130_mixed", dict(batch=3, n=130, cond=2, seed=141, case="mixed")),
]

# Blocked compact-WY prototype runs: (name, spec, panel_width)
BLOCKED = [
    ("blk_8_p3", dict(batch=3, n=8, cond=1, seed=321), 3),
    ("blk_40_p8", dict(batch=2, n=40, cond=2, seed=322, case="mixed"), 8),
]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the fast-qr checkout")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "official"))
    sys.path.insert(0, str(ref / "tools"))
    from reference import check_implementation, generate_input  # type: ignore
    from blocked_qr_reference import blocked_geqrf_reference  # type: ignore

    assert not torch.cuda.is_available(), "fixtures are generated on CPU"
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, dict] = {"cases": {}, "blocked": {}, "torch": torch.__version__}
    for name, spec in SPECS:
        a = generate_input(**spec)
        h32, t32 = torch.geqrf(a.clone())
        h64, t64 = torch.geqrf(a.double())
        ok, msg = check_implementation(a, (h32, t32))
        arrays[f"{name}.A"] = a.numpy()
        arrays[f"{name}.H32"] = h32.contiguous().numpy()
        arrays[f"{name}.tau32"] = t32.numpy()
        arrays[f"{name}.H64"] = h64.contiguous().numpy()
        arrays[f"{name}.tau64"] = t64.numpy()
        meta["cases"][name] = {"spec": spec, "official_ok": bool(ok), "official_message": msg}
    for name, spec, pw in BLOCKED:
        a = generate_input(**spec)
        hb, tb = blocked_geqrf_reference(a, panel_width=pw, update_mode="compact-wy")
        ok, msg = check_implementation(a, (hb, tb))
        arrays[f"{name}.A"] = a.numpy()
        arrays[f"{name}.H"] = hb.contiguous().numpy()
        arrays[f"{name}.tau"] = tb.numpy()
        meta["blocked"][name] = {"spec": spec, "panel_width": pw, "official_ok": bool(ok),
                                 "official_message": msg}
    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(arrays)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
