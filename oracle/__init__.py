"""CPU oracle for the TabPack packed-ensemble hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (`tabpack_b200`) imports this
package; only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` /
`--impl reference` legs of `bench.py` may use it, and there only as the checker
or as the timed CPU restatement of the reference.

Every function restates the reference algorithm (Abusagit/tabpack,
`src/tabpackage/*.py`) in numpy and cites the file:line it follows.  The
restatement is pinned against golden vectors produced by running the reference
itself (`tests/golden/make_golden.py`), see `tests/test_oracle_golden.py`.
"""
