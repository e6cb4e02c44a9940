"""CPU oracle for the trispconv sparse-convolution hot path.

TEST INFRASTRUCTURE ONLY.  This package restates, in numpy, the algorithm of
the reference's pure-PyTorch CPU path (mrpulford/trispconv,
``trispconv/pytorch/indices.py``, ``functional.py``, ``modules.py``,
``weight.py``).  It is the checker for the CUDA library: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product package ``trispconv_b200``
never imports or calls anything here.

Parity pins: ``tests/test_oracle_golden.py`` checks this restatement against
(a) the nine spconv-2.x golden fixtures shipped with the reference
(``tests/fixtures/spconv_golden_*.pt``, converted to ``tests/golden/*.npz``)
and (b) pair tables and outputs produced by the reference itself
(``tests/golden/make_golden.py``).
"""
from oracle.indices import (  # noqa: F401
    OracleIndiceData,
    encode_coords,
    inverse_pairs,
    output_spatial_shape,
    strided_pairs,
    subm_pairs,
    to3,
)
from oracle.conv import conv_forward, normalize_weight  # noqa: F401
from oracle.network import network_kmaps, run_layers  # noqa: F401
