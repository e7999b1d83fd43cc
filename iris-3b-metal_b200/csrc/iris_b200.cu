// Single translation unit of libiris_b200.so: the device error word and the
// kernels share one module, so no relocatable device code is needed.
#include "abi.cu"
#include "adapter.cu"
#include "attention.cu"
#include "gemm.cu"
#include "heads.cu"
#include "peer.cu"
#include "pixel.cu"
#include "rows.cu"
#include "small.cu"
#include "tiles.cu"
