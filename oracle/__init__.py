"""Test oracle for the FlowEdge policy-sampling hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (`flowedge_b200/`, the
C-ABI library) imports, links or runs anything in this directory.  Only
`tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg use it,
and only as the checker / the timed CPU baseline.

* `restate.py`  - numpy restatement of the reference algorithm, each function
  citing the reference file:line it follows.
* `reference.py` - ctypes binding to `_ref/liboracle.so`, the reference's own
  C++ core compiled from its sources by `Makefile` (parity is pinned against
  it and against the golden fixtures under tests/golden/).
"""
