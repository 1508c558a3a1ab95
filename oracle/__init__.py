"""CPU oracle for the op pass -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline arm may
import this package; the product (thintnpu_b200 / libttn.so) never does, and
it has no CPU fallback.  The oracle is PyTorch CPU eager on the same fp16
inputs (FP32 compute rounded to fp16 per op), which is the parity contract of
the path, plus a numpy restatement of the reference's stable selection order
(verify_selection_flow.py:27-93, selection_flow.cpp:30-57 and 322-366).

Pinning: ``tests/test_oracle.py`` checks the selection restatement against
golden outputs of the reference's own CPU restatement (``reference()`` in
verify_selection_flow.py) on its 47 fixtures and the exhaustive 65,536-half
key/float-bits checks; the elementwise/layout oracles are the reference
tests' own CPU formulas (verify_flow_ops.py:13-35, verify_softmax.py,
verify_dfl_softmax.py, verify_ops.py, verify_all.py).
"""
