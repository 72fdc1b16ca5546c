"""tq_mla: B200-native absorbed MLA attention over a paged latent KV cache.

The compute path is libtq_mla.so (hand-written CUDA for sm_100a behind the C ABI of
``include/tq_mla.h``); this package is the host-side mirror of the reference's operator
interface. Importing ``tq_mla.ops`` loads the library and fails loudly if it was not built.
"""

__version__ = "0.1.0"
