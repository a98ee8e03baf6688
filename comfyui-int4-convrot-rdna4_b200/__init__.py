"""B200 (sm_100a) ConvRot W4A4 backend for the ComfyUI-INT4-ConvRot node package.

``_int4`` is the drop-in backend package (same public API as the node's own
``_int4``); ``csrc`` holds the CUDA kernels and the C ABI.
"""
