"""Per-request logits dumps written by the coordinator (`serve --export-logits DIR`).

Parity: rust/src/distributed/coordinator.rs:358-388 (`write_raw_logits_file`,
`export_logits_dump`) and its callers (:1170-1190 prefill, :1336-1368 continuation, :2208-2240 the
continuation end-to-end run). The layout is the reference's so its comparison scripts read both:
one directory per request, one `<name>.f32le` file per artifact (the vocabulary's logits as raw
little-endian float32, no header) and a `meta.json` describing the run. A failed write is logged
and never fails the request.
"""

from __future__ import annotations

import json
import logging
import os
from typing import Dict, Mapping

import numpy as np
import torch

log = logging.getLogger("hcp.logits_dump")


def write_raw_logits(path: str, logits) -> None:
    a = logits.detach().float().cpu().numpy() if isinstance(logits, torch.Tensor) else np.asarray(logits)
    a.astype("<f4").reshape(-1).tofile(path)


def read_raw_logits(path: str) -> np.ndarray:
    return np.fromfile(path, dtype="<f4")


def export_logits_dump(out_dir: str, artifacts: Mapping[str, object], meta: Dict) -> bool:
    """Write `artifacts` (name -> 1-D logits) and `meta.json` into `out_dir`; True on success."""
    try:
        os.makedirs(out_dir, exist_ok=True)
        for name, logits in artifacts.items():
            write_raw_logits(os.path.join(out_dir, f"{name}.f32le"), logits)
        with open(os.path.join(out_dir, "meta.json"), "w") as f:
            json.dump(meta, f, indent=2)
        return True
    except (OSError, ValueError) as e:
        log.warning("logits export to %s failed: %s", out_dir, e)
        return False


def argmax(logits) -> int:
    t = logits if isinstance(logits, torch.Tensor) else torch.as_tensor(np.asarray(logits))
    return int(torch.argmax(t.float().view(-1)))
