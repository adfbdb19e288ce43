// Single translation unit of libgdn_b200.so: the device error word and every kernel
// live in one module, so no relocatable device code or device link step is needed.
#include "capi.cu"
#include "recurrent.cu"
#include "verify_block.cu"
#include "conv.cu"
#include "norm.cu"
#include "chunk.cu"
#include "noalloc.cu"
#include "gates.cu"
#include "attention.cu"
#include "rotary.cu"
#include "probe.cu"
#include "inproj.cu"
