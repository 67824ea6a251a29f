"""qsa_b200 -- B200-native (sm_100a) sparse paged GQA FP8 decode attention.

A drop-in for the decode-attention path of Ammar-Alnagar/QSA-FP8-SM89: the
same torch-callable contract (``run``, ``launch``, ``qsa_decode``), backed by
hand-written sm_100a CUDA kernels behind a C ABI (``include/qsa_b200.h``,
``libqsa_b200.so``) and a thin ``torch.ops.qsa_b200`` extension over it.
"""

from ._lib import QsaBuildError, load_clib, load_torch_ops
from .ops import launch, qsa_cache_write, qsa_decode, qsa_topk_select, run, slots, token_slots, workspace_bytes

__all__ = [
    "QsaBuildError",
    "launch",
    "load_clib",
    "load_torch_ops",
    "qsa_cache_write",
    "qsa_topk_select",
    "qsa_decode",
    "run",
    "slots",
    "token_slots",
    "workspace_bytes",
]
