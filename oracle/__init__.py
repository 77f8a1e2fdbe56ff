"""CPU oracle for the 12-bit-codec decode path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference algorithms (karabilo214/AI, `ramvi/engine/ramvi_engine/...`), each
function citing the reference file:line it follows. It is pinned against golden vectors produced by the
reference itself (`tests/golden/make_golden.py` runs the reference codec, its Triton kernels under the
interpreter and its Numba CPU code; the fixtures are committed under `tests/golden/`).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm may import this
package, and only as the checker. The product (`ai_b200`) never imports it and has no CPU fallback.
"""
