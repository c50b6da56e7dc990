"""CPU oracle for TurboPolar's compressed-KV decode path (TEST INFRASTRUCTURE ONLY).

This package restates, in NumPy, the algorithm of the reference's CPU path for the hot
path (dawsonblock/Turbopolar, which runs it on MLX):

* ``oracle.polar``   -- polar key codec, ``rfsn_v11/quant/polar/encoder.py:24-130`` and
  ``rfsn_v11/quant/polar/decoder.py:7-85``;
* ``oracle.vquant``  -- grouped int8 value codec, ``rfsn_v11/quant/v_quant/encoder.py:16-38``;
* ``oracle.attention`` -- the bridge's CPU fallbacks ``_cpu_fused_qk`` /
  ``_cpu_online_attention`` / ``_cpu_online_attention_dense_tail``
  (``rfsn_v11/kernels/turbo_polar/metal.py:254-332``), evaluated in float64;
* ``oracle.runtime`` -- the cache runtime's tail / flush / telemetry bookkeeping,
  ``rfsn_v11/generation/turbo_polar_cache.py:55-395`` with the storage growth of
  ``rfsn_v11/generation/storage.py:17-169``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and only as the checker: the product (``turbopolar_b200``) never calls it and
fails loudly when its CUDA library is missing.

Parity pin: the fixtures in ``tests/golden/`` were produced by executing the reference's own
Python sources (unmodified) over a NumPy stand-in for ``mlx.core``
(``tests/golden/mlx_standin``), because MLX cannot be installed here.  The oracle is
checked against every fixture (``tests/test_oracle_golden.py``).  What the fixtures pin is
the reference's code path: packing order, layout, split of level-1/deep codes, flush and
tail logic, byte accounting, fallback attention.  They do NOT pin MLX's own float16
transcendental rounding: both the stand-in and this oracle model MLX's float32 ``atan2``,
``log``, ``exp``, ``sin``, ``cos`` as correctly rounded (float64 evaluation rounded to
float32), so bit-level code parity against real MLX execution is unpinned.
"""

from . import polar, vquant, attention, runtime  # noqa: F401
