"""CPU oracle for the segmented separation forward.

TEST INFRASTRUCTURE ONLY. Nothing in the ``unblend_b200`` package imports this
package: it is the checker that ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` run beside the CUDA
path, never the thing measured or shipped.

* ``htdemucs_oracle`` restates ``HTDemucs.forward`` (unblend/htdemucs.py:650-704)
  with plain fp32 torch CPU ops over a reference-layout ``state_dict``.
* ``apply_oracle`` restates the overlapping-segment loop of
  ``apply_model_multi`` (unblend/apply.py:567-1333) for shifts 0 and >0.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference itself
(weights from ``torch.manual_seed``, synthetic audio) and committed its outputs
as fixtures; ``tests/test_oracle.py`` checks this restatement against them.
"""
