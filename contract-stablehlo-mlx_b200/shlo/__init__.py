"""Host-side mirror of the StableHLO executor's device layer, over libshlo_cuda.

The reference's host is Lean (StablehloMlx/*.lean); its toolchain is not
available here, so this package restates the Lean layers that sit right above
the FFI boundary, one module each, with the reference's names:

  mlx    StablehloMlx/Mlx.lean          the 25 @[extern] entry points, op codes, dtypes
  run    StablehloMlx/Kernels/Run.lean  kernel cache, parameter words, one wrapper per kernel
  lower  StablehloMlx/Lower.lean        the op table's call sequences and planted faults
  exec   StablehloMlx/Exec.lean         load / prepare / call, with a generic-form reader

Every device operation goes through the C ABI of include/shlo_cuda.h. There
is no CPU fallback: importing `mlx` (and so `run`, `lower`, `exec`)
loads the CUDA library and fails if it is missing. Two modules are host-only
and load nothing: `denoiser` (the benchmark workload as module text, weights
and inputs) and `shard` (the partition rules and host collectives), so a
CPU-only caller such as the CPU baseline can use them without mapping the
CUDA library.
"""
