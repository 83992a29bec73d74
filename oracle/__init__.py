"""CPU oracle for the per-layer weight-quantization hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may use it, and only as the checker (or as the timed
CPU baseline), never as a code path of the product.

``cpu_ref`` restates, in numpy/scipy fp32 arithmetic, the reference
implementation of ThunderFun/int_crush_converter (``converter/*.py``).  Every
function cites the reference file:line it follows.  The restatement is pinned
against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``, fixtures in ``tests/golden/golden.npz``).
"""
