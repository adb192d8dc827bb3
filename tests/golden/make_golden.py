"""Generate the golden fixtures in this directory from the reference itself.

Run where the dgx-monarch source tree is readable, naming its `src`
directory by argument or by the DGXM_REFERENCE_SRC environment variable:

    python tests/golden/make_golden.py <dgx-monarch>/src

It imports the reference's own in-repo USP modules (adapters/base.py,
usp_full_axis.py, usp_pad_exclusion.py, usp_sequence_order.py,
cfg_parallel.py, cudnn_ring_attention.py) with xfuser / yunchang replaced by
stubs in sys.modules, exactly where the reference's tests place theirs
(tests/test_usp_full_axis.py:12-27, tests/test_usp_pad_exact.py:323-360), and
records inputs and outputs as small fixtures.  Nothing at test time reads the
reference; the tests compare the oracle (oracle/usp.py) with these files.
"""
from __future__ import annotations

import json
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch

REF_SRC: Path | None = None  # the dgx-monarch `src` directory, set by main()


def _reference_src(argv: list[str]) -> Path:
    """The reference's `src` directory from the first argument or
    DGXM_REFERENCE_SRC; it must hold the dgx_monarch package."""
    import os

    given = argv[1] if len(argv) > 1 else os.environ.get("DGXM_REFERENCE_SRC")
    if not given:
        raise SystemExit("usage: make_golden.py <dgx-monarch src directory> "
                         "(or set DGXM_REFERENCE_SRC)")
    src = Path(given).resolve()
    if not (src / "dgx_monarch" / "adapters" / "base.py").exists():
        raise SystemExit(f"{src} does not hold dgx_monarch/adapters/base.py")
    return src
OUT = Path(__file__).resolve().parent


# Kernel options handed to the Wan Ring2 ring function (flash's surface).
_FLASH_DEFAULTS = {"dropout_p": 0.0, "softmax_scale": None, "causal": False, "window_size": (-1, -1),
                   "softcap": 0.0, "alibi_slopes": None, "return_softmax": False}
FLASH_SURFACE_CASES = [dict(_FLASH_DEFAULTS, **change) for change in (
    {}, {"softmax_scale": 0.125}, {"softmax_scale": 1}, {"dropout_p": 0}, {"softcap": 0},
    {"dropout_p": 0.1}, {"dropout_p": False}, {"dropout_p": float("nan")}, {"dropout_p": "0"},
    {"softmax_scale": 0.0}, {"softmax_scale": -1.0}, {"softmax_scale": float("inf")},
    {"softmax_scale": True}, {"causal": True}, {"causal": 0}, {"window_size": [-1, -1]},
    {"window_size": (-1, 0)}, {"window_size": (-1, -1, -1)}, {"window_size": (True, -1)},
    {"softcap": 30.0}, {"softcap": float("-inf")}, {"alibi_slopes": "slopes"},
    {"return_softmax": True}, {"return_softmax": 0},
)]

# Local shards: (shape q, shape k, shape v, dtype, requires_grad, layout).
LOCAL_QKV_CASES = [
    {"q": [1, 8, 2, 128], "k": [1, 8, 2, 128], "v": [1, 8, 2, 128], "dtype": "bfloat16"},
    {"q": [1, 8, 2, 128], "k": [1, 8, 2, 128], "v": [1, 8, 2, 128], "dtype": "bfloat16", "grad": True},
    {"q": [8, 2, 128], "k": [8, 2, 128], "v": [8, 2, 128], "dtype": "bfloat16"},
    {"q": [1, 8, 2, 128], "k": [1, 8, 2, 128], "v": [1, 9, 2, 128], "dtype": "bfloat16"},
    {"q": [1, 8, 3, 128], "k": [1, 8, 2, 128], "v": [1, 8, 2, 128], "dtype": "bfloat16"},
    {"q": [1, 0, 2, 128], "k": [1, 0, 2, 128], "v": [1, 0, 2, 128], "dtype": "bfloat16"},
    {"q": [1, 8, 2, 128], "k": [1, 8, 2, 128], "v": [1, 8, 2, 128], "dtype": "float32"},
    {"q": [1, 8, 2, 128], "k": [1, 8, 2, 128], "v": [1, 8, 2, 128], "dtype": "float16"},
    {"q": [1, 8, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64], "dtype": "bfloat16"},
    {"q": [1, 8, 2, 128], "k": [1, 16, 2, 128], "v": [1, 16, 2, 128], "dtype": "bfloat16"},
]


# Ring block-processor calls (adapters/cudnn_ring_attention.py:26-89): kernel
# options, then q/k/v shapes and dtypes; on CPU tensors a well-formed call
# ends at the CUDA-device refusal.
RING_PROCESSOR_CASES = [
    {"kw": {}},
    {"kw": {"softmax_scale": 0.125}},
    {"kw": {"softmax_scale": 1}},
    {"kw": {"softmax_scale": 0.0}},
    {"kw": {"softmax_scale": -1.0}},
    {"kw": {"softmax_scale": {"float": "inf"}}},
    {"kw": {"softmax_scale": True}},
    {"kw": {"softmax_scale": "0.1"}},
    {"kw": {"dropout_p": 0.1}},
    {"kw": {"causal": True}},
    {"kw": {"window_size": {"tuple": [0, 0]}}},
    {"kw": {"alibi_slopes": "slopes"}},
    {"kw": {"softcap": 1.0}},
    {"kw": {"return_softmax": True}},
    {"kw": {"deterministic": True}},
    {"kw": {"block_mask": None}},
    {"q": [1, 8, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64], "dtype": "float32"},
    {"q": [8, 2, 64], "k": [8, 2, 64], "v": [8, 2, 64]},
    {"q": [1, 0, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64]},
    {"q": [1, 8, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64], "grad": True},
    {"q": [1, 8, 3, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64]},
    {"q": [1, 8, 2, 64], "k": [1, 8, 2, 64], "v": [1, 9, 2, 64]},
    {"q": [1, 8, 2, 64], "k": [2, 8, 2, 64], "v": [2, 8, 2, 64]},
    {"q": [1, 5, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64], "dtype": "float16"},
    {"q": [1, 8, 2, 64], "k": [1, 8, 2, 64], "v": [1, 8, 2, 64], "dtype": "float16", "k_dtype": "bfloat16"},
]


# Per-cond CFG dispatch (adapters/cfg_dispatch.py:92-206): conditioning
# slots described as lists of entries -- text tokens, an optional batch
# constant and optional unmodelled keys, hooks or a control object name --
# built into comfy-like cond objects by build_cond_slots below (the test
# builds the same objects).
COND_FOLD_CASES = [
    {"slots": [[{"tokens": 7}], [{"tokens": 7}]]},
    {"slots": [[{"tokens": 7}], [{"tokens": 11}]]},
    {"slots": [[{"tokens": 2}], [{"tokens": 8}]]},
    {"slots": [[{"tokens": 77}], [{"tokens": 154}]]},
    {"slots": [[{"tokens": 100}], [{"tokens": 28}]]},
    {"slots": [[{"tokens": 7, "const": 9}], [{"tokens": 7, "const": 11}]], "key": "num_tokens"},
    {"slots": [[{"tokens": 7, "const": 9}], [{"tokens": 11, "const": 9}]], "key": "num_tokens"},
    {"slots": [[{"tokens": 7}], [{"tokens": 11, "area": True}]]},
    {"slots": [[{"tokens": 7, "hooks": "h"}], [{"tokens": 11}]]},
    {"slots": [[{"tokens": 7, "control": "a"}], [{"tokens": 11, "control": "b"}]]},
    {"slots": [[{"tokens": 7}], None]},
    {"slots": [[{"tokens": 7}], [{"tokens": 11}], [{"tokens": 13}]]},
    {"slots": [[{"tokens": 7}, {"tokens": 7}], [{"tokens": 7}]]},
    {"slots": [[{"tokens": 7, "extra": True}], [{"tokens": 7}]]},
]


class _FakeCrossAttn:
    """A comfy CONDCrossAttn-like object: its length rule decides can_concat."""

    def __init__(self, tokens):
        self.cond = torch.zeros(1, tokens, 4)

    def process_cond(self, batch_size, area):
        return self

    def can_concat(self, other):
        a, b = self.cond.shape[1], other.cond.shape[1]
        if a == b:
            return True
        lo, hi = min(a, b), max(a, b)
        return lo > 0 and math.lcm(lo, hi) // lo <= 4


class _FakeConstant:
    def __init__(self, value):
        self.cond = value

    def process_cond(self, batch_size, area):
        return self

    def can_concat(self, other):
        return self.cond == other.cond


def build_cond_slots(case):
    controls = {}
    slots = []
    for slot in case["slots"]:
        if slot is None:
            slots.append(None)
            continue
        entries = []
        for e in slot:
            conds = {"c_crossattn": _FakeCrossAttn(e["tokens"])}
            if "const" in e:
                conds["num_tokens"] = _FakeConstant(e["const"])
            if e.get("extra"):
                conds["y"] = object()  # a cond without comfy's methods
            item = {"model_conds": conds, "control": controls.setdefault(e.get("control"), object())
                    if e.get("control") else None}
            if e.get("area"):
                item["area"] = (1, 1, 0, 0)
            if e.get("hooks"):
                item["hooks"] = e["hooks"]
            entries.append(item)
        slots.append(entries)
    return slots


# Malformed (and two well-formed) usp_attention calls: tensor shapes, the
# call's keyword arguments, and an optional mask ("effective" or "noop").
USP_REFUSAL_CASES = [
    {"q": [1, 8, 64], "k": [1, 8, 64], "v": [1, 8, 64], "kw": {"heads": 4}},
    {"q": [1, 8, 100], "k": [1, 8, 100], "v": [1, 8, 100], "kw": {"heads": 3}},
    {"q": [1, 8, 64], "k": [1, 8, 64], "v": [1, 8, 64], "kw": {"heads": 4, "skip_reshape": True}},
    {"q": [1, 2, 8, 16], "k": [1, 2, 8, 16], "v": [1, 2, 8, 16], "kw": {"heads": 4, "skip_reshape": True}},
    {"q": [1, 2, 8, 16], "k": [2, 2, 8, 16], "v": [1, 2, 8, 16], "kw": {"heads": 2, "skip_reshape": True}},
    {"q": [1, 2, 8, 16], "k": [1, 2, 8, 16], "v": [1, 2, 8, 16], "kw": {"heads": 2}},
    {"q": [1, 8, 32], "k": [2, 8, 32], "v": [1, 8, 32], "kw": {"heads": 2}},
    {"q": [1, 8, 32], "k": [1, 8, 40], "v": [1, 8, 40], "kw": {"heads": 2}},
    {"q": [1, 8, 32], "k": [1, 8, 32], "v": [1, 8, 16], "kw": {"heads": 2}},
    {"q": [1, 8, 64], "k": [1, 8, 32], "v": [1, 8, 32], "kw": {"heads": 4}},
    {"q": [1, 8, 48], "k": [1, 8, 32], "v": [1, 8, 32], "kw": {"heads": 3, "enable_gqa": True}},
    {"q": [1, 8, 64], "k": [1, 8, 64], "v": [1, 8, 64], "kw": {"heads": 4}, "mask": "effective"},
    {"q": [1, 8, 64], "k": [1, 8, 64], "v": [1, 8, 64], "kw": {"heads": 4}, "mask": "noop"},
]


def build_usp_call(case: dict):
    """CPU tensors and keyword arguments of a usp_attention case."""
    q, k, v = (torch.zeros(case[n]) for n in "qkv")
    kwargs = dict(case["kw"])
    if case.get("mask") == "effective":
        mask = torch.zeros(1, 1, 8, 8)
        mask[..., 0] = -1e9
        kwargs["mask"] = mask
    elif case.get("mask") == "noop":
        kwargs["mask"] = torch.zeros(1, 1, 8, 8)
    return q, k, v, kwargs


def encode_case(case: dict) -> dict:
    """JSON form of a kernel-option case: tuples, non-finite floats and the
    bool/int distinction survive (tests/test_full_context_host.py decodes)."""
    def enc(x):
        if isinstance(x, tuple):
            return {"tuple": [enc(y) for y in x]}
        if isinstance(x, list):
            return {"list": [enc(y) for y in x]}
        if isinstance(x, float) and not math.isfinite(x):
            return {"float": repr(x)}
        return x
    return {key: enc(value) for key, value in case.items()}


def _decode_case(x):
    """Inverse of encode_case for one value."""
    if isinstance(x, dict):
        if set(x) == {"tuple"}:
            return tuple(_decode_case(y) for y in x["tuple"])
        if set(x) == {"list"}:
            return [_decode_case(y) for y in x["list"]]
        if set(x) == {"float"}:
            return float(x["float"])
    return x


def build_qkv(case: dict):
    """CPU tensors of a local-shard case."""
    dt = getattr(torch, case["dtype"])
    q, k, v = (torch.zeros(case[n], dtype=dt) for n in "qkv")
    if case.get("grad"):
        q.requires_grad_(True)
    return q, k, v


def _install_stubs(ring_world=1, gathered=None, world=1, rank=0):
    """The xfuser / yunchang leaves, as the reference's tests stub them."""
    calls = []

    class AllToAll:
        @staticmethod
        def apply(_group, tensor, scatter, gather):
            calls.append((scatter, gather, tensor.detach().clone()))
            if (scatter, gather) == (2, 1) and gathered is not None:
                return gathered.to(dtype=tensor.dtype)
            return tensor

    class StubUSP:
        ulysses_pg = ring_pg = attn_type = attn_processor = None
        q_descale = k_descale = v_descale = None

        def __init__(self, *args, **kwargs):
            pass

        def __call__(self, attn, q_l, k_l, v_l, **kwargs):
            return _attend64(q_l, k_l, v_l)

        @staticmethod
        def ring_attn_fn(q, k, v, **kwargs):
            return _attend64(q, k, v)

    mods = {name: types.ModuleType(name) for name in (
        "xfuser", "xfuser.core", "xfuser.core.distributed", "xfuser.core.long_ctx_attention",
        "yunchang", "yunchang.kernels", "yunchang.comm", "yunchang.comm.all_to_all")}
    mods["xfuser.core.distributed"].get_ring_parallel_world_size = lambda: ring_world
    mods["xfuser.core.distributed"].get_sequence_parallel_world_size = lambda: world
    mods["xfuser.core.distributed"].get_sequence_parallel_rank = lambda: rank
    mods["xfuser.core.long_ctx_attention"].xFuserLongContextAttention = StubUSP
    mods["yunchang.kernels"].AttnType = {"TORCH_FLASH": "TORCH_FLASH"}
    mods["yunchang.comm.all_to_all"].SeqAllToAll4D = AllToAll
    sys.modules.update(mods)
    return calls, StubUSP


def _attend64(q, k, v):
    """float64 softmax(q k^T / sqrt(D)) v in (B, L, H, D), the reference tests' kernel."""
    qh, kh, vh = (t.transpose(1, 2).double() for t in (q, k, v))
    scores = qh @ kh.transpose(-1, -2) / math.sqrt(qh.shape[-1])
    return (torch.softmax(scores, dim=-1) @ vh).transpose(1, 2).to(q.dtype)


def _full_context_rank(rank, port, k, v, out_q, ref_src):
    """One gloo rank running the reference's Ring2 K/V gather
    (adapters/wan_ring_full_context.py:203-295)."""
    import os

    import torch.distributed as dist

    sys.path.insert(0, str(ref_src))
    _install_stubs()
    from dgx_monarch.adapters.wan_ring_full_context import _materialize_full_kv_batch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    full_k, full_v = _materialize_full_kv_batch(k[rank], v[rank], group=None, world=2, rank=rank,
                                                global_ranks=(0, 1))
    out_q.put((rank, full_k.numpy(), full_v.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def _full_context_golden(rng, arrays) -> list:
    """Run the reference's full-context gather on a world-2 gloo group."""
    import socket

    import torch.multiprocessing as mp

    cases = []
    for n, (length, heads, dim) in enumerate(((5, 2, 4), (3, 1, 8))):
        k = [torch.from_numpy(rng.standard_normal((1, length, heads, dim))) for _ in range(2)]
        v = [torch.from_numpy(rng.standard_normal((1, length, heads, dim))) for _ in range(2)]
        with socket.socket() as sock:
            sock.bind(("127.0.0.1", 0))
            port = sock.getsockname()[1]
        ctx = mp.get_context("spawn")
        out_q = ctx.Queue()
        procs = [ctx.Process(target=_full_context_rank, args=(r, port, k, v, out_q, str(REF_SRC))) for r in range(2)]
        for proc in procs:
            proc.start()
        got = dict((r, (fk, fv)) for r, fk, fv in (out_q.get(timeout=120) for _ in range(2)))
        for proc in procs:
            proc.join(timeout=60)
        for r in range(2):
            arrays[f"fullctx_{n}_k{r}"] = k[r].numpy()
            arrays[f"fullctx_{n}_v{r}"] = v[r].numpy()
            arrays[f"fullctx_{n}_fullk{r}"] = got[r][0]
            arrays[f"fullctx_{n}_fullv{r}"] = got[r][1]
        cases.append({"index": n, "length": length, "heads": heads, "dim": dim})
    return cases


def main() -> None:
    global REF_SRC
    REF_SRC = _reference_src(sys.argv)
    sys.path.insert(0, str(REF_SRC))
    _install_stubs()
    import dgx_monarch.adapters.base as base
    from dgx_monarch.adapters import cfg_parallel, cudnn_ring_attention
    from dgx_monarch.adapters.usp_full_axis import run_full_axis
    from dgx_monarch.adapters.usp_pad_exclusion import keep_index
    from dgx_monarch.adapters.usp_sequence_order import RankMajorJointOrder

    golden: dict = {}
    arrays: dict[str, np.ndarray] = {}
    rng = np.random.default_rng(2026)

    # a) gathered pad-row coordinates (adapters/base.py:134-149), including the
    #    hand-computed Krea2 geometries of tests/test_usp_pad_exact.py:28-75.
    cases = [([(512, 256), (9216, 4608)], 2), ([(512, 256), (8281, 4141)], 2),
             ([(511, 256), (8281, 4141)], 2), ([(512, 256), (8275, 4139)], 2),
             ([(510, 128), (8281, 2071)], 4), ([(511, 511), (8281, 8281)], 1),
             ([(511, 256)], 2), ([(512, 256)], 2)]
    for _ in range(24):
        world = int(rng.choice([2, 3, 4, 8]))
        segs = []
        for _s in range(int(rng.integers(1, 4))):
            orig = int(rng.integers(1, 5000))
            segs.append((orig, -(-orig // world)))
        cases.append((segs, world))
    padded = []
    for segs, world in cases:
        base.sp_world = (lambda w=world: w)
        padded.append({"segments": segs, "world": world, "rows": base.padded_row_indices(segs)})
    golden["padded_row_indices"] = padded

    # b) joint key order (adapters/usp_sequence_order.py:69-146).
    joint = []
    for text, image, world in ((1, 1, 2), (3, 5, 2), (128, 2048, 2), (7, 2, 4), (64, 1152, 8),
                               (2, 4, 2), (5, 3, 3)):
        order = RankMajorJointOrder(text, image)
        rows = world * (text + image)
        perm = order.permutation(rows, torch.device("cpu")).tolist()
        drop = sorted(set(int(x) for x in rng.integers(0, rows, size=min(4, rows))))
        kv_drop = sorted(set(int(x) for x in rng.integers(0, rows, size=min(3, rows))))
        z = torch.zeros(1, rows, 1, 1)
        _q, _k, _v, qd, kd, _p = order.canonicalize(z, z, z, drop, kv_drop, None)
        joint.append({"text": text, "image": image, "world": world, "permutation": perm,
                      "drop": drop, "kv_drop": kv_drop, "canon_drop": qd, "canon_kv_drop": kd})
    golden["joint_order"] = joint

    # c) keep index (adapters/usp_pad_exclusion.py:79-126).
    keeps = []
    for rows, drop in ((6, []), (4, [1]), (14, [5, 13]), (10, [8, 9]), (4, [3]), (9728, [4652, 8793])):
        idx = keep_index(rows, drop, torch.device("cpu"))
        keeps.append({"rows": rows, "drop": drop, "kept": None if idx is None else idx.tolist()})
    golden["keep_index"] = keeps

    # d) the full-axis Ulysses composition with an order descriptor and pads
    #    (adapters/usp_full_axis.py:9-40), float64, the rank-major gathered axis
    #    handed in the way tests/test_usp_full_axis.py:67-91 does.
    full = []
    for n, (text, image, world, hds, dim, drop, kvdrop) in enumerate(
            ((2, 2, 2, 2, 3, [3], [7]), (3, 5, 2, 2, 4, [7, 15], [2, 11]), (2, 4, 3, 1, 8, [], []))):
        rows = world * (text + image)
        gathered = torch.from_numpy(rng.standard_normal((1, rows, hds, dim)))
        calls, usp_cls = _install_stubs(gathered=gathered)
        out = run_full_axis(usp_cls(), gathered[:, :rows // world], gathered[:, :rows // world],
                            gathered[:, :rows // world], drop, kvdrop, None,
                            RankMajorJointOrder(text, image), None)
        arrays[f"full_axis_{n}_in"] = gathered.numpy()
        arrays[f"full_axis_{n}_sent"] = calls[-1][2].numpy()  # what the inverse all-to-all got
        arrays[f"full_axis_{n}_out"] = out.numpy()
        full.append({"index": n, "text": text, "image": image, "world": world,
                     "drop": drop, "kv_drop": kvdrop})
    golden["full_axis"] = full

    # e) the usp_attention callable at world 1 (adapters/base.py:216-326):
    #    reshape surfaces, GQA repeat_interleave, pad-row exclusion.
    _install_stubs()
    attn = base._make_usp_attention_callable(sys.modules["xfuser.core.long_ctx_attention"]
                                             .xFuserLongContextAttention())
    callable_cases = []
    specs = [
        dict(b=1, l=10, h=4, hkv=4, d=8, skip=False, gqa=False, drop=None),
        dict(b=2, l=7, h=4, hkv=2, d=8, skip=False, gqa=True, drop=None),
        dict(b=1, l=14, h=4, hkv=4, d=8, skip=True, gqa=False, drop=[5, 13]),
        dict(b=1, l=9, h=2, hkv=1, d=16, skip=True, gqa=True, drop=[8]),
    ]
    for n, s in enumerate(specs):
        q = torch.from_numpy(rng.standard_normal((s["b"], s["l"], s["h"], s["d"])))
        k = torch.from_numpy(rng.standard_normal((s["b"], s["l"], s["hkv"], s["d"])))
        v = torch.from_numpy(rng.standard_normal((s["b"], s["l"], s["hkv"], s["d"])))
        if s["skip"]:
            out = attn(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), heads=s["h"],
                       skip_reshape=True, skip_output_reshape=True, enable_gqa=s["gqa"],
                       drop_rows=s["drop"]).transpose(1, 2)
        else:
            out = attn(q.reshape(s["b"], s["l"], -1), k.reshape(s["b"], s["l"], -1),
                       v.reshape(s["b"], s["l"], -1), heads=s["h"], enable_gqa=s["gqa"],
                       drop_rows=s["drop"]).reshape(s["b"], s["l"], s["h"], s["d"])
        for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
            arrays[f"callable_{n}_{name}"] = t.numpy()
        callable_cases.append({"index": n, **s})
    golden["usp_callable"] = callable_cases

    # f) the CFG batch slice (adapters/cfg_parallel.py:71-87).
    x = rng.standard_normal((4, 3, 2))
    bcast = rng.standard_normal((1, 3))
    tree = {"x": torch.from_numpy(x), "nested": [torch.from_numpy(x[:, 0]), torch.from_numpy(bcast)]}
    slices = []
    for world in (2, 4):
        for rank in range(world):
            sl = cfg_parallel._take_slice(tree, 4, world, rank)
            arrays[f"cfg_{world}_{rank}_x"] = sl["x"].numpy()
            arrays[f"cfg_{world}_{rank}_n0"] = sl["nested"][0].numpy()
            arrays[f"cfg_{world}_{rank}_n1"] = sl["nested"][1].numpy()
            slices.append({"world": world, "rank": rank})
    arrays["cfg_in_x"], arrays["cfg_in_bcast"] = x, bcast
    golden["cfg_slice"] = slices

    # g) shard_seq chunks (adapters/base.py:91-123).
    t = rng.standard_normal((1, 7, 3))
    shards = []
    for world in (2, 3, 4):
        for rank in range(world):
            base.sp_world = (lambda w=world: w)
            base.sp_rank = (lambda r=rank: r)
            local, orig = base.shard_seq(torch.from_numpy(t))
            arrays[f"shard_{world}_{rank}"] = local.numpy()
            shards.append({"world": world, "rank": rank, "orig": orig})
    arrays["shard_in"] = t
    golden["shard_seq"] = shards

    # h) the dyadic known-answer probe of the cuDNN ring processor
    #    (adapters/cudnn_ring_attention.py:106-135): record its inputs and the
    #    expected (out, lse) its own formula computes, in fp32 on the CPU.
    seen = []

    def recorder(q, k, v, softmax_scale=None):
        qh, kh, vh = (value.transpose(1, 2).float() for value in (q, k, v))
        scores = torch.matmul(qh, kh.transpose(-1, -2)) * softmax_scale
        lse = torch.logsumexp(scores, dim=-1)
        out = torch.matmul(torch.softmax(scores, dim=-1), vh).transpose(1, 2).to(q.dtype)
        seen.append((q.clone(), k.clone(), v.clone(), out.clone(), lse.clone(), softmax_scale))
        return out, lse

    cudnn_ring_attention._probe_native(recorder, device=torch.device("cpu"))
    for n, (q, k, v, out, lse, scale) in enumerate(seen):
        for name, tt in (("q", q), ("k", k), ("v", v), ("out", out)):
            arrays[f"probe_{n}_{name}"] = tt.float().numpy()
        arrays[f"probe_{n}_lse"] = lse.numpy()
    golden["probe"] = [{"index": n, "dtype": str(s[0].dtype), "scale": s[5]} for n, s in enumerate(seen)]

    # i) query-group biases through the usp_attention callable at world 1
    #    (adapters/base.py:299-316 -> usp_full_axis.py:14-16 ->
    #    usp_query_bias.py:109-130), comfy's SDPA wrapper stubbed by torch SDPA
    #    as tests/test_usp_query_bias.py:26-29 passes it: the LTX guide
    #    rectangles (one weight, per-token weights with a zero), a Lens-style
    #    single key-bias group, a per-head bias, and a padded stream whose tail
    #    pads are dropped (tests/test_usp_query_bias.py:198-223).
    comfy = types.ModuleType("comfy")
    comfy_ops = types.ModuleType("comfy.ops")
    comfy_ops.scaled_dot_product_attention = (
        lambda q, k, v, attn_mask=None: torch.nn.functional.scaled_dot_product_attention(
            q, k, v, attn_mask=attn_mask))
    sys.modules.update({"comfy": comfy, "comfy.ops": comfy_ops})
    _install_stubs()
    attn = base._make_usp_attention_callable(sys.modules["xfuser.core.long_ctx_attention"]
                                             .xFuserLongContextAttention())

    def guide(tokens, guide_start, weights):
        finfo = torch.finfo(weights.dtype)
        log_w = torch.full_like(weights, finfo.min)
        log_w[weights > 0] = torch.log(weights[weights > 0])
        tracked = weights.shape[0]
        noisy = torch.zeros((1, 1, 1, tokens), dtype=weights.dtype)
        noisy[..., guide_start:guide_start + tracked] = log_w.view(1, 1, 1, -1)
        rect = torch.zeros((1, 1, tracked, tokens), dtype=weights.dtype)
        rect[..., :guide_start] = log_w.view(1, 1, -1, 1)
        groups = [(0, guide_start, noisy), (guide_start, guide_start + tracked, rect)]
        if guide_start + tracked < tokens:
            groups.append((guide_start + tracked, tokens, None))
        return groups

    f64 = torch.float64
    bias_cases = [
        ("ltx_uniform", 12, 4, guide(12, 8, torch.full((4,), 0.7, dtype=f64)), None),
        ("ltx_pixel", 14, 4, guide(14, 9, torch.tensor([0.2, 0.8, 0.0, 1.0, 0.55], dtype=f64)), None),
        ("ltx_partial", 16, 2, guide(16, 9, torch.full((4,), 0.3, dtype=f64)), None),
        ("lens_key_bias", 11, 2, [(0, 11, torch.from_numpy(rng.standard_normal((1, 1, 1, 9))))], None),
        ("per_head", 10, 2, [(0, 4, None), (4, 10, torch.from_numpy(rng.standard_normal((1, 2, 1, 10))))],
         None),
        ("padded_tail", 14, 4, guide(12, 8, torch.full((4,), 0.7, dtype=f64)), [12, 13]),
    ]
    biased = []
    for name, tokens, hds, groups, drop in bias_cases:
        q = torch.from_numpy(rng.standard_normal((1, hds, tokens, 8)))
        k = torch.from_numpy(rng.standard_normal((1, hds, tokens, 8)))
        v = torch.from_numpy(rng.standard_normal((1, hds, tokens, 8)))
        out = attn(q, k, v, heads=hds, skip_reshape=True, skip_output_reshape=True,
                   drop_rows=drop, query_bias_groups=tuple(groups))
        for key, t in (("q", q), ("k", k), ("v", v), ("out", out)):
            arrays[f"bias_{name}_{key}"] = t.transpose(1, 2).numpy()
        spec = []
        for g, (start, end, bias) in enumerate(groups):
            if bias is not None:
                arrays[f"bias_{name}_g{g}"] = bias.numpy()
            spec.append([start, end, None if bias is None else f"bias_{name}_g{g}"])
        biased.append({"name": name, "tokens": tokens, "heads": hds, "groups": spec, "drop": drop})
    golden["query_bias"] = biased

    # j) the Wan Ring2 full-context K/V gather on a world-2 gloo group: the
    #    rank-major slots every rank's local-Q x full-KV call reads.
    golden["full_context"] = _full_context_golden(rng, arrays)

    # k) the shared NVFP4 activation scale (adapters/quant_activation_scale.py:
    #    222-246) with a replay reducer standing in for the max all-reduce, as
    #    tests/test_nvfp4_shard_scale.py:165-178 runs it: every shard of one
    #    tensor must get the scale one GPU takes over the whole tensor.
    from dgx_monarch.adapters import quant_activation_scale as qas

    scales = []
    for n, (dtype, world, rows, cols, outlier) in enumerate((
            (torch.bfloat16, 2, 64, 64, 30.0), (torch.bfloat16, 4, 96, 40, -7.25),
            (torch.float16, 2, 32, 48, 11.0), (torch.float32, 3, 30, 20, 5.5),
            (torch.bfloat16, 8, 128, 256, 0.0))):
        x = torch.from_numpy(rng.standard_normal((rows, cols)).astype(np.float32)).to(dtype)
        if outlier:
            x[rows - 3, cols // 2] = outlier
        shards = torch.chunk(x, world, dim=0)
        local = [sh.abs().amax().to(torch.float32).reshape(1) for sh in shards]
        shared = torch.stack(local).amax(dim=0)
        plan = qas.SharedScalePlan((("sp", lambda t, m=shared: torch.maximum(t, m)),))
        got = [qas.shared_activation_scale(sh, plan, qas.NVFP4_SCALE_DIVISOR) for sh in shards]
        arrays[f"scale_{n}_x"] = x.to(torch.float32).numpy()
        arrays[f"scale_{n}_out"] = torch.stack([g.to(torch.float32) for g in got]).numpy()
        scales.append({"index": n, "dtype": str(dtype).replace("torch.", ""), "world": world,
                       "divisor": qas.NVFP4_SCALE_DIVISOR})
    golden["shared_scale"] = scales

    # l) the Wan Ring2 full-context refusals (adapters/wan_ring_full_context.py:
    #    17-117): every kernel option and local-shard case below, with the
    #    reference's verdict -- accepted, or its refusal message.
    from dgx_monarch.adapters import wan_ring_full_context as wfc

    def verdict(fn, **kwargs):
        try:
            fn(**kwargs)
            return "ok"
        except base.UnsupportedModelError as exc:
            return str(exc)

    surface = []
    for case in FLASH_SURFACE_CASES:
        surface.append({"case": encode_case(case),
                        "verdict": verdict(wfc._validate_flash_surface, **case)})
    qkv = []
    for case in LOCAL_QKV_CASES:
        q, k, v = build_qkv(case)
        qkv.append({"case": case, "verdict": verdict(wfc._validate_local_qkv, q=q, k=k, v=v)})
    golden["full_context_surface"] = surface
    golden["full_context_qkv"] = qkv

    # m) the usp_attention callable's typed refusals (adapters/base.py:216-292):
    #    each malformed call below with the reference's verdict.
    _install_stubs()
    attn = base._make_usp_attention_callable(sys.modules["xfuser.core.long_ctx_attention"]
                                             .xFuserLongContextAttention())
    refusals = []
    for case in USP_REFUSAL_CASES:
        q, k, v, kwargs = build_usp_call(case)
        try:
            attn(q, k, v, **kwargs)
            said = "ok"
        except base.UnsupportedModelError as exc:
            said = str(exc)
        refusals.append({"case": case, "verdict": said})
    golden["usp_refusals"] = refusals

    # n) the cuDNN ring block processor's verdicts on those calls.
    processor = cudnn_ring_attention.TorchCudnnRingProcessor()
    ring_verdicts = []
    for case in RING_PROCESSOR_CASES:
        dt = getattr(torch, case.get("dtype", "bfloat16"))
        shapes = [case.get(n, [1, 8, 2, 64]) for n in "qkv"]
        q, k, v = (torch.zeros(shape, dtype=dt) for shape in shapes)
        if "k_dtype" in case:
            k = k.to(getattr(torch, case["k_dtype"]))
        if case.get("grad"):
            q.requires_grad_(True)
        kwargs = {key: _decode_case(value) for key, value in case.get("kw", {}).items()}
        try:
            processor(q, k, v, **kwargs)
            said = "ok"
        except base.UnsupportedModelError as exc:
            said = str(exc)
        ring_verdicts.append({"case": case, "verdict": said})
    golden["ring_processor"] = ring_verdicts

    # o) per-cond CFG dispatch: the fold verdicts, the cond groups and the
    #    cross-attention length rule of adapters/cfg_dispatch.py.
    from dgx_monarch.adapters import cfg_dispatch

    x_in = torch.zeros(2, 3)
    golden["cond_fold"] = [{"case": case, "folds": bool(cfg_dispatch.conds_fold(
        build_cond_slots(case), x_in, case.get("key")))} for case in COND_FOLD_CASES]
    golden["cond_groups"] = [{"count": c, "world": w, "rank": r,
                              "bounds": list(cfg_dispatch.cond_group_bounds(c, w, r))}
                             for c in range(0, 7) for w in (1, 2, 3, 4, 8) for r in range(w)]
    golden["cross_attn_folds"] = [{"a": a, "b": b, "folds": cfg_dispatch.cross_attn_pair_folds(a, b)}
                                  for a in (0, 1, 2, 7, 11, 28, 44, 77, 100, 154, 256, 512)
                                  for b in (0, 1, 2, 8, 11, 44, 77, 154, 300, 512)]

    (OUT / "golden.json").write_text(json.dumps(golden, indent=1))
    np.savez_compressed(OUT / "golden_arrays.npz", **arrays)
    print("wrote", OUT / "golden.json", OUT / "golden_arrays.npz")


if __name__ == "__main__":
    main()
