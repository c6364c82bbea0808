"""Token sampling: greedy, temperature, nucleus (top-p).

Parity: rust/src/model/sampling.rs:8-119 (greedy when temperature == 0, else softmax(logits / T),
top-p by sorted cumulative probability, multinomial draw). Runs on whatever device the logits are
on; the coordinator samples on rank 0 and ships the chosen id to every rank with the next command,
so all ranks stay in lock step.
"""

from __future__ import annotations

from typing import Optional

import torch


def sample_token(logits: torch.Tensor, temperature: float = 0.0, top_p: float = 1.0,
                 generator: Optional[torch.Generator] = None) -> int:
    logits = logits.float().view(-1)
    if temperature <= 0.0:
        return int(torch.argmax(logits))
    probs = torch.softmax(logits / float(temperature), dim=-1)
    if 0.0 < top_p < 1.0:
        sp, idx = torch.sort(probs, descending=True)
        cum = torch.cumsum(sp, dim=-1)
        keep = cum - sp < top_p          # always keeps the most likely token
        sp = sp * keep
        sp = sp / sp.sum()
        choice = torch.multinomial(sp, 1, generator=generator)
        return int(idx[choice])
    return int(torch.multinomial(probs, 1, generator=generator))
