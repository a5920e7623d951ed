"""Record the reference UNet's state-dict layout (names, shapes, dtypes) as a fixture.

Runs in the development container only (needs the reference checkout):

    python tests/golden/make_unet_keys.py /path/to/reference

The test suite compares fp8_b200.unet.UNet against this file, so checkpoints
move between the two models without conversion.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = Path(__file__).resolve().parent


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    import torch
    from diffusion.unet import UNet, UNetConfig  # the reference module

    out = {}
    for name, attn in (("attn16", [16]), ("attn16_8", [16, 8])):
        cfg = UNetConfig(3, base_hidden=128, scales=[1, 2, 2, 2], n_heads=4, p_drop=0.1, attn_resolutions=attn,
                         in_resolution=32, n_resblocks=2, fp8_convs_enabled=True, fp8_scaling_type="delayed")
        torch.manual_seed(0)
        model = UNet(cfg)
        out[name] = {
            "params": sum(p.numel() for p in model.parameters()),
            "state_dict": [[k, list(v.shape), str(v.dtype)] for k, v in model.state_dict().items()],
        }
    path = HERE / "reference_unet_state_dict.json"
    path.write_text(json.dumps(out))
    print(f"wrote {path}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <checkout of the reference repository>")
    main(sys.argv[1])
