"""Tolerance rules shared by the model-level parity tests (GPU vs oracle, HF vs oracle).

Logits: 2e-2 relative error.  Greedy ids: equal, except at near-ties.  On
identical inputs a near-tie is a row whose two largest oracle logits are within
2 bf16 ulps; after steps on a KV cache whose bf16 rows differ from the oracle's
by rounding (or against a float32 forward), a mismatch is allowed when the
oracle logits of the two tokens differ by at most the logits tolerance (2e-2 of
the row's largest magnitude) or 2 bf16 ulps."""

import numpy as np
import torch


def near_tie(logits: torch.Tensor) -> torch.Tensor:
    top2 = torch.topk(logits, 2, dim=-1).values
    ulp = 2.0 ** (torch.floor(torch.log2(top2[:, 0].abs().clamp_min(1e-30))) - 7)
    return (top2[:, 0] - top2[:, 1]) <= 2 * ulp


def within_logit_tol(ref_row: torch.Tensor, dev_id: int) -> tuple[bool, str]:
    """A greedy mismatch after decoding on a device's own KV cache: allowed when
    the oracle logits of its token and of the device's token differ by less
    than the logits tolerance (2e-2 of the row's largest magnitude) or by at
    most 2 bf16 ulps."""
    top = int(torch.argmax(ref_row))
    gap = float(ref_row[top] - ref_row[dev_id])
    scale = float(ref_row.abs().max())
    ulp = 2.0 ** (np.floor(np.log2(max(abs(float(ref_row[top])), 1e-30))) - 7)
    return gap <= max(2e-2 * scale, 2 * ulp), f"gap {gap:.4g}, row scale {scale:.4g}, ulp {ulp:.3g}"
