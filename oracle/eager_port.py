"""CPU port of the reference's eager PyTorch path, for the timed CPU baseline.

TEST INFRASTRUCTURE ONLY. ``bench.py`` times this on the GPU box's host cores
(its ``cpu_baseline`` leg and its ``--impl reference`` arm); the tests use it
as a second check of the numpy oracle. It is never on the product path.

The reference's ``torch_eager`` (sm89_torch.py:27-54) reads its shapes from
module globals (``NUM_REQUESTS``, ``TOPK``, ``MAX_PAGES`` ...) that
``sm89_cutedsl`` fixes at import. This port takes them from the tensors
instead and otherwise runs the same ATen operator sequence:

1. index decode with the ``0 <= t < context`` mask (sm89_torch.py:30-34),
   where the context is ``pages_per_req * P`` (the reference's ``TOPK``);
2. block-table gather with the ``0 <= phys < num_pages`` mask (:36-39);
3. advanced-index gather of K/V and the cast to float32 (:43-44);
4. ``matmul`` QK scaled by ``k_scale / sqrt(D)`` (:45-47);
5. ``masked_fill(-inf)`` and ``softmax`` (:48-49);
6. ``matmul`` PV scaled by ``v_scale`` (:50);
7. sigmoid gate and the bf16 cast (:51-54).

Like the reference it ignores any count column and gives NaN for a row
without a valid token.
"""

from __future__ import annotations

import math

import torch


@torch.inference_mode()
def torch_eager_port(q, k, v, k_scale, v_scale, btable, t2r, indices, gate):
    rows, hq, d = q.shape
    num_pages, page_size, hkv, _ = k.shape
    nreq, pages_per_req = btable.shape
    context = pages_per_req * page_size
    grp = hq // hkv

    logical = indices[:, :context].to(torch.long)
    valid = (logical >= 0) & (logical < context)
    logical = logical.clamp(0, context - 1)
    logical_page = logical // page_size
    page_offset = logical % page_size

    request_ids = t2r.to(torch.long).clamp(0, nreq - 1)
    physical_page = btable[request_ids[:, None], logical_page]
    valid &= (physical_page >= 0) & (physical_page < num_pages)
    physical_page = physical_page.clamp(0, num_pages - 1)

    keys = k[physical_page, page_offset].permute(0, 2, 3, 1).to(torch.float32)
    values = v[physical_page, page_offset].permute(0, 2, 1, 3).to(torch.float32)
    queries = q.reshape(rows, hkv, grp, d).float()

    scores = torch.matmul(queries, keys) * (k_scale / math.sqrt(d))
    scores = scores.masked_fill(~valid[:, None, None, :], -torch.inf)
    probabilities = torch.softmax(scores, dim=-1)
    context_v = torch.matmul(probabilities, values) * v_scale
    gated = context_v * torch.sigmoid(gate.reshape(rows, hkv, grp, d).float())
    return gated.reshape(rows, hq, d).to(torch.bfloat16)
