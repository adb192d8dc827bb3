"""CPU oracle for the sequence-parallel attention path.

TEST INFRASTRUCTURE ONLY.  This package restates, on the CPU, the algorithm the
reference (dgx-monarch) runs on its attention seam, so the CUDA path can be
checked against it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import it, and only as the checker or the timed CPU baseline;
nothing in dgx_monarch_b200/ imports it, and the product path fails loudly
rather than falling back to it.

Parity pinning: every integer/permutation function is checked against golden
vectors produced by running the reference's own in-repo modules
(tests/golden/make_golden.py) and against the hand-computed layouts in the
reference's tests.  The third-party leaves the reference calls (yunchang
SeqAllToAll4D and ring attention, xfuser group getters) are absent; their
conventions are restated from the reference's stubs and call sites.
"""
