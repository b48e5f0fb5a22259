"""CPU oracle for the paged fused-MoE path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and
``bench.py``'s CPU-baseline / reference arm use it.

* ``oracle.pager``    - restatement of the reference LRU pager
  (``WispMoEState.ensure_resident``) and of the first-fit token sub-batching
  of the paged forward; pinned against golden traces recorded from the
  reference itself (``tests/golden/``).
* ``oracle.setorder`` - the CPython set-iteration-order model that decides
  the reference's slot placement.
* ``oracle.moe``      - fp32 restatement of the per-(token, expert) FFN and
  the routing-order combine that vLLM's ``fused_experts`` computes for the
  reference.
"""
