"""kestrel_b200: a B200 (sm_100a) backend for Kestrel's Mixture-of-Experts FFN.

`kestrel_b200.cuda` binds the C ABI of libkestrel_cuda.so
(include/kestrel_cuda.h); `kestrel_b200.ggml` holds the GGML block-format
table and this project's deterministic quantizer; `kestrel_b200.build`
compiles the CUDA library in-tree.
"""
