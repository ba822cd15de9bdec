"""furykernel-cuda: a B200-native (sm_100a) target for FuryKernel programs.

- `furykernel_b200.target`: the target's caps and its `Backend` (`cuda`).
- `furykernel_b200._native`: the C ABI of libfurykernel_cuda.so
  (include/furykernel_cuda.h): contexts, buffers, checked launches, graphs.
- `furykernel_b200.shape`: the Llama-shaped model's shape.
- `furykernel_b200._host`: the C ABI of libfurykernel_host.so
  (include/furykernel_host.h): programs, plans and launch lists.
- `furykernel_b200.engine`, `prefill`, `tp`: the decode step, the prompt
  prefill and tensor parallelism on the device.
"""

__version__ = "0.1.0"
