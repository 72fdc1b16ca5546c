"""Oracle package: CPU restatements of the reference's algorithms, used only as test checkers.

Modules: ``philox`` (Philox4x32-10 stream), ``generate`` (seeded synthetic inputs), ``mla``
(float64 absorbed MLA core and its paged dense extension), ``contracts`` (SMLA host contract),
``schedule`` (the split-KV work partition, restated for the bit-exact metadata check).
The product never imports this package; its CUDA path fails loudly if the extension is absent.
"""
