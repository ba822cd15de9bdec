"""furykernel-cuda: a B200-native (sm_100a) target for FuryKernel programs.

- `furykernel_b200.target`: the target's caps and its `Backend` (`cuda`).
- `furykernel_b200._native`: the C ABI of libfurykernel_cuda.so
  (include/furykernel_cuda.h): contexts, buffers, checked launches, graphs.
- `furykernel_b200.program`: programs, their gate and the planner, restated
  from the reference's program layer.
- `furykernel_b200.engine`: the launch sequence of a plan on the device.
"""

__version__ = "0.1.0"
