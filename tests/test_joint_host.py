"""Host-side checks of the replicated-text joint attention (no GPU): the
argument refusals run before any device work.  The data path itself is
checked on the GPU (tests/test_ulysses_gpu.py, tests/test_multigpu.py) and
its CPU restatement over gloo in tests/test_gloo_usp.py."""
from __future__ import annotations

import pytest
import torch


@pytest.mark.parametrize("kwargs,needle", [
    ({"world": 3, "heads": 8, "head_dim": 64}, "do not divide"),
    ({"world": 2, "heads": 8, "head_dim": 130}, "head_dim 130"),
    ({"world": 2, "heads": 8, "head_dim": 60}, "head_dim 60"),
    ({"world": 2, "heads": 8, "head_dim": 64, "seq_local": 0}, "image row"),
    ({"world": 2, "heads": 8, "head_dim": 64, "txt_rows": -1}, "text length"),
])
def test_joint_refuses_bad_geometry_before_device_work(kwargs, needle):
    from dgx_monarch_b200.ulysses import JointUlyssesAttention

    args = {"rank": 0, "batch": 1, "seq_local": 16, "txt_rows": 4, "device": torch.device("cpu")}
    args.update(kwargs)
    with pytest.raises(ValueError, match=needle):
        JointUlyssesAttention(**args)



class _RecordingLib:
    """Stands in for libdgxm_sp.so: records the joint scatter's arguments."""

    def __init__(self):
        self.calls = []

    def dgxm_ulysses_scatter_joint(self, desc, txt_rows, txt_front, txt, strides, src, dst, stream):
        d = desc._obj
        self.calls.append({"txt_rows": txt_rows, "txt_front": txt_front, "seq_local": d.seq_local,
                           "heads": d.heads, "world": d.world, "rank": d.rank,
                           "strides": list(strides) if txt_rows else None})
        return 0


class _Stream:
    cuda_stream = 0


@pytest.mark.parametrize("text,text_first", [(0, True), (5, True), (7, False)])
def test_joint_scatter_passes_the_text_rows_it_was_given(monkeypatch, text, text_first):
    """The text row count comes from the text tensors only (0 without text),
    never from the image tensors; strides are the text tensors' own."""
    from dgx_monarch_b200 import _lib, ulysses

    rec = _RecordingLib()
    monkeypatch.setattr(_lib, "load", lambda: rec)
    monkeypatch.setattr(ulysses, "_require_cuda", lambda *t: None)
    img = [torch.zeros(1, 12, 4, 16, dtype=torch.bfloat16) for _ in range(3)]
    txt = [torch.zeros(1, 2 * text, 4, 16, dtype=torch.bfloat16)[:, ::2] for _ in range(3)] if text else None
    ulysses.ulysses_scatter_joint(img, txt, [[0, 0] for _ in range(3)], world=2, rank=1,
                                  text_first=text_first, stream=_Stream())
    (call,) = rec.calls
    assert call["txt_rows"] == text and call["txt_front"] == int(text_first)
    assert (call["seq_local"], call["heads"], call["world"], call["rank"]) == (12, 4, 2, 1)
    if text:
        assert call["strides"] == [x for t in txt for x in (t.stride(0), t.stride(1), t.stride(2))]
    with pytest.raises(ValueError):
        ulysses.ulysses_scatter_joint(img, [torch.zeros(1, 3, 4, 8, dtype=torch.bfloat16)] * 3,
                                      [[0, 0] for _ in range(3)], world=2, rank=1, stream=_Stream())


def test_joint_scatter_refuses_host_tensors():
    """Host pointers never reach a kernel: the wrappers refuse CPU tensors."""
    from dgx_monarch_b200 import ulysses

    img = [torch.zeros(1, 4, 2, 16, dtype=torch.bfloat16) for _ in range(3)]
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ulysses.ulysses_scatter_joint(img, None, [[0] for _ in range(3)], world=1, rank=0, stream=_Stream())
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        ulysses.ulysses_scatter(img, [[0] for _ in range(3)], world=1, rank=0, stream=_Stream())


def test_device_checks_skip_absent_tensors_and_refuse_host_ones():
    from dgx_monarch_b200.ops import _require_cuda, _require_on, check_attn_buffers

    assert _require_cuda() is None and _require_cuda(None, None) is None
    _require_on(torch.device("cuda", 0), None, None)
    _require_on("cuda:1")
    host = torch.zeros(2, 3)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _require_cuda(None, host)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _require_on(torch.device("cuda", 0), host)
    q = torch.zeros(1, 4, 2, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        check_attn_buffers(q, q, out=torch.zeros(1, 4, 2, 8))

