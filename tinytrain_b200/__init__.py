"""tinytrain_b200: tinytrain's training hot path on B200 (sm_100a).

The compute lives in two in-tree shared libraries built by
`python -m tinytrain_b200.build`:
  lib/libttk.so        CUDA kernels behind the C ABI of include/ttk.h
  lib/libtinytrain.so  the C++20 tt:: Tensor/ops/nn/optim/model API on device
                       storage, plus the trainer C ABI of include/tt_trainer.h
"""
__all__ = ["build", "kernels", "trainer"]
