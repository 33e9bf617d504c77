"""torch_kunlun for B200: the int16-quantised dense-op hot path of torch_kunlun
(mm / linear / addmm / bmm / baddbmm / matmul / conv2d, softmax, layer_norm,
SDPA and the bkcl collectives) rebuilt on hand-written sm_100a kernels."""

__version__ = "0.1.0"
