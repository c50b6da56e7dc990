"""B200-native TurboPolar compressed-KV decode path.

Public API (names of dawsonblock/Turbopolar):

* :class:`TurboPolarConfig` -- supported-configuration contract
* :class:`TurboPolarKVCacheRuntime` -- ``append / attention / get_io_telemetry / reset`` with
  the page store on the GPU
* :class:`CudaKernelBridge` -- the bridge's ``execute_*`` calls
* :class:`PolarQuantEncoder`, :class:`PolarQuantDecoder`, :class:`GroupedVQuantizer`
* :mod:`turbopolar_b200.llama` -- PyTorch Llama adapter (``TurboPolarFastCache``,
  ``make_turbo_caches``, ``patch_llama_attention``)
* :mod:`turbopolar_b200.sharded` -- sequence-sharded multi-GPU attention

All compute runs in ``libturbopolar.so`` (``include/turbopolar.h``), built by
``python -m turbopolar_b200.build``.
"""

from .config import TurboPolarConfig
from .payload import PolarKeyBlock, QuantizedVBlock
from .cache import TurboPolarKVCacheRuntime
from .codec import GroupedVQuantizer, PolarQuantDecoder, PolarQuantEncoder
from .bridge import CudaKernelBridge

__all__ = [
    "TurboPolarConfig", "TurboPolarKVCacheRuntime", "CudaKernelBridge", "PolarKeyBlock", "QuantizedVBlock",
    "PolarQuantEncoder", "PolarQuantDecoder", "GroupedVQuantizer",
]
