"""CPU oracle for the uTTT serving hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's fast-weight operator, its
analytical chunk-TTT write and the frozen/updating model forward of
Phova/uTTTCompanion (``model/uttt_layer.py``, ``model/uttt_model.py``).  Every
function cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline /
reference arm may import it, and only as the checker or the timed CPU
baseline.  The product package (``utttcompanion_b200``) never imports it and
has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` runs the reference implementation
itself (importable on the development host) on seeded inputs and stores the
outputs as ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this
oracle against those fixtures (FP64 to 1e-10, FP32 to 1e-5, BF16-autocast
emulation to BF16 rounding noise).
"""

from . import numerics, fastweight, model  # noqa: F401
