// fp4x_all.cu -- single translation unit of libfp4x.so (the device error word
// and the kernels share one module without relocatable device code).
#include "api.cu"
#include "quant.cu"
#include "gemv.cu"
#include "elementwise.cu"
#include "attention.cu"
#include "mma.cu"
#include "persist.cu"
#include "persist_tc.cu"
#include "tp.cu"
#include "engine.cu"
#include "loader.cu"
#include "batch.cu"
