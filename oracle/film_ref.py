"""fp32 restatement of FrameResidualQueryFiLMAdapter (test oracle).

Follows duplex_kernel/frame_residual_adapter.py:156-237 (``residual`` :203-234,
``forward`` :236-237) and apply_response_state_residual's frame-0 rule
(:55-71, ``preserve_frame0``).  Weights use the adapter's state_dict names.
TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


@torch.no_grad()
def film_forward(w: dict[str, torch.Tensor], hidden: torch.Tensor, query: torch.Tensor,
                 max_scale: float = 0.25) -> torch.Tensor:
    """query + tanh(output(fused)) * scale * RMS(query), all in fp32."""
    w = {k: v.float() for k, v in w.items()}
    q_in = query.float()
    h_in = hidden.float()
    qn = F.layer_norm(q_in, (q_in.shape[-1],), w["query_norm.weight"], w["query_norm.bias"], 1e-5)
    qd = qn @ w["query_down.weight"].t() + w["query_down.bias"]
    rn = F.layer_norm(h_in, (h_in.shape[-1],), w["response_norm.weight"], w["response_norm.bias"], 1e-5)
    rd = F.silu(rn @ w["response_down.weight"].t() + w["response_down.bias"])
    film = rd @ w["film.weight"].t() + w["film.bias"]
    gamma, beta = film.chunk(2, dim=-1)
    fused = F.silu(qd * (1.0 + torch.tanh(gamma)) + beta)
    mapped = fused @ w["output.weight"].t() + w["output.bias"]
    amp = torch.sqrt(torch.mean(q_in.square(), dim=-1, keepdim=True))
    scale = max_scale * torch.sigmoid(w["scale_logit"])
    return q_in + torch.tanh(mapped) * scale * amp
