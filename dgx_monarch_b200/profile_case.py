"""Run one attention shape three times, for profiler captures.

    python -m dgx_monarch_b200.profile_case SEQ HEADS
"""
import sys

import torch

from dgx_monarch_b200.ops import attention_fwd

seq, heads = (int(sys.argv[1]), int(sys.argv[2])) if len(sys.argv) > 2 else (32768, 8)
g = torch.Generator(device="cuda").manual_seed(0)
q, k, v = (torch.randn(1, seq, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
out = torch.empty_like(q)
for _ in range(3):
    attention_fwd(q, k, v, out=out, return_lse=False)
torch.cuda.synchronize()
