"""Record the reference mHC modules' checkpoint layout: for each module class
and a few (n, C), the state_dict keys with shape and dtype, and the values of
the parameters whose initialisation is deterministic (gate scales and
biases).  A checkpoint written by the reference trainer (a state_dict, saved in
fp16 by trainer/train_pretrain.py:63-71) loads into this build's modules only
if these match.  Imports the reference from ``--reference`` (a read-only
checkout) and writes tests/golden/state_layout.json::

    python tests/golden/make_state_layout.py --reference /path/to/minimind-mhc
"""

from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a read-only checkout of the reference")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from model.mhc_common import MHCHead, StreamExpand
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres

    out = {}
    for cls in (MHCConnection_Fused, MHCConnection_FusedNoHres, MHCHead, StreamExpand):
        for n, c in ((4, 768), (2, 512), (4, 1024)):
            torch.manual_seed(0)
            m = cls(n, c)
            entries = {}
            for k, v in m.state_dict().items():
                e = {"shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")}
                if not k.startswith("phi"):
                    e["value"] = v.reshape(-1).tolist()
                entries[k] = e
            out[f"{cls.__name__}/{n}/{c}"] = entries
    with open(os.path.join(HERE, "state_layout.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
