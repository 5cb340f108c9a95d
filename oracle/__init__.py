"""CPU oracle for the CSA/HCA decode path over a TurboQuant paged KV cache.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
package; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg do, and only as the checker (or, in ``bench.py``, as the
timed CPU restatement of the reference's own torch path).

Every function restates an algorithm of the reference project
(itz-sayak/deepseek-v4-codebase) in float32 torch CPU arithmetic -- the same
arithmetic library and op order the reference uses -- and cites the file:line
it follows.  Parity of this restatement with the reference itself is pinned
by ``tests/golden/*.npz`` (written by ``tests/golden/make_golden.py``, which
imports the reference) and checked in ``tests/test_oracle_golden.py``.
"""
