// q3_dispatch.cu -- the six IREE-substitution kernels as one standalone
// sm_100a object, for the route of compile.sh:47-66: each
// iree/dispatch_N.mlir wrapper names this object, and iree-compile embeds it
// in place of the executable decode_dispatch_N of model/qwen3_full.mlir.
// The kernels are those of libq3b200.so (csrc/q3_iree.cuh): same export
// names, parameter lists and fixed launch (grid N/8 x 256 threads).
#include "../csrc/q3_iree.cuh"
