"""CPU oracle for the FlashUMA eSCN/UMA message-passing hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline. The product path
(``flash_uma_b200``) never imports it and has no CPU fallback.

Contents
* ``oracle.ops``   - PyTorch (CPU) restatement of the six reference ops, forward
  differentiable so ``torch.autograd`` gives the reference's backward.
* ``oracle.model`` - restatement of ``model.py`` (Morton reorder, CSR, layer loop)
  and ``wrapper.py`` (weight transfer, csd embedding, shifts).

Pinning: the restatement is checked against golden vectors produced by running
the reference's own Triton ops on CPU (``tests/golden/make_golden.py``); see
``tests/test_oracle_golden.py``.
"""
