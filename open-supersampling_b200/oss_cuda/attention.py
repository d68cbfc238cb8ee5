"""Cross-attention entry point kept for import compatibility.

The reference ships this as an unimplemented stub (oss/cuda/oss_cuda/attention.py:7-11);
it is outside the rasterizer path, so it stays a stub here too.
"""


def fused_window_cross_attention(*args, **kwargs):
    raise NotImplementedError(
        "fused_window_cross_attention is not part of the B200 rasterizer library; "
        "use the PyTorch cross-attention path."
    )
