"""CPU restatement of the batched Control6 policy head (test oracle).

Follows NativeControl6LoRA.forward (training/duplex_qlora/native_control6.py:
157-197) -- the frozen six LM-head rows applied in the rows' dtype (bf16) and
widened, plus the rank-r LoRA delta on [hidden ; phase] in fp32 -- and the
per-batch selection of GemmaNativeControl6BatchPolicy.step_batch
(duplex_kernel/gemma_native_control6_batch_policy.py:878-893): raw argmax,
argmax over the legal actions, its softmax probability among the legal
logits, and the finite check.  TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

ACTIONS = 6
HIDDEN = 1536
PHASE = 4


@torch.no_grad()
def control6_head(hidden: torch.Tensor, phase: torch.Tensor | None, legal: torch.Tensor,
                  base_rows: torch.Tensor, lora_a: torch.Tensor, lora_b: torch.Tensor,
                  scaling: float) -> tuple[torch.Tensor, torch.Tensor]:
    """hidden [n,1536] (bf16), phase [n,4] or None, legal bool [n,6] ->
    (logits f32 [n,6], packet f32 [n,4] = finite, raw, selected, confidence)."""
    n = hidden.shape[0]
    h32 = hidden.float()
    ph = torch.zeros(n, PHASE) if phase is None else phase.float()
    base = F.linear(hidden.to(base_rows.dtype), base_rows).float()
    delta = F.linear(F.linear(torch.cat((h32, ph), dim=-1), lora_a.float()), lora_b.float()) * scaling
    logits = base + delta
    finite = torch.isfinite(logits).all(dim=1).float()
    raw = logits.argmax(dim=1)
    selected_logits = logits.masked_fill(~legal, -torch.inf)
    sel = selected_logits.argmax(dim=1)
    conf = torch.softmax(selected_logits, dim=1).gather(1, sel[:, None])[:, 0]
    return logits, torch.stack((finite, raw.float(), sel.float(), conf), dim=1)
