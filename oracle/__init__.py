"""CPU oracle of ASPIRE's unified mixed forward hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ``aspire_b200``
package) imports this package; only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` may use it, as the checker and as
the timed CPU reference, never as a code path of the GPU product.

Modules:

* ``oracle.attention``     - paged mixed draft/verify attention and the
                             first/last logit dump (fp32 torch restatement of
                             FlashInfer's semantics as ASPIRE drives them).
* ``oracle.page_selector`` - restatement of PageSelectorFirstLastAvg and
                             _store_draft_rows.
* ``oracle.kv_append``     - restatement of mylib::update_kv_padded.

Pinning: ``tests/golden/`` holds fixtures produced by the reference's own
code (its PageSelectorFirstLastAvg and HostPlanState imported from the
reference tree, its Triton append kernel run by Triton's CPU interpreter);
``tests/test_oracle_golden.py`` checks this restatement against them.  The
attention restatement is pinned against the semantics of FlashInfer's
persistent kernel source (see ``oracle/attention.py``).
"""
