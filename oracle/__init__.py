"""CPU oracle for the DSA hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the algorithms of the reference operators
(18851871668/dsa_triton_ascend) so the CUDA kernels in ``dsa_triton_ascend_b200``
can be checked against them on the same seeded inputs.

Rules for this package:

* Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
  ``--impl reference`` legs of ``bench.py`` may import it, and only as the checker
  or as the timed CPU baseline. The product path (``dsa_triton_ascend_b200``) never
  imports it and has no CPU fallback.
* Every function cites the reference ``file:line`` it restates.

Pinning status (see ``tests/test_oracle_golden.py``):

* ``sfa.sfa_fwd``  -- pinned against ``sparse_flash_attention_numpy.py`` goldens.
* ``sfa.sfa_bwd``  -- pinned against ``sparse_flash_attention_grad_numpy.py`` goldens.
* ``sli.sli_grad`` -- pinned against ``sli_grad_kl_loss_numpy.py`` goldens (run with
  its fp16 emulation switched on; the fp32 mode is the kernel-faithful default).
* ``li.li_score`` / ``li.li_topk`` -- **parity unpinned**: the reference ships no
  golden for the lightning indexer (its only check is against closed CANN
  kernels), so this restatement of ``lightning_indexer_triton.py:202-280, 339-357``
  is checked only by hand-computed known-answer cases.
"""
