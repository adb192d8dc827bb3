"""Drive one attention shape three times (for ncu captures): argv = seq heads."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import torch  # noqa: E402

from dgx_monarch_b200.ops import attention_fwd  # noqa: E402

seq, heads = (int(sys.argv[1]), int(sys.argv[2])) if len(sys.argv) > 2 else (32768, 8)
g = torch.Generator(device="cuda").manual_seed(0)
q, k, v = (torch.randn(1, seq, heads, 128, device="cuda", generator=g).bfloat16() for _ in range(3))
out = torch.empty_like(q)
for _ in range(3):
    attention_fwd(q, k, v, out=out, return_lse=False)
torch.cuda.synchronize()
