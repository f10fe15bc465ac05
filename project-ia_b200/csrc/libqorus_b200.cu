// libqorus_b200.cu — the single translation unit of libqorus_b200.so.
// The kernels are header-defined and included once here, so no relocatable
// device code (and no device link step) is needed.
#include "runtime.cu"
#include "tp.cu"
#include "model.cu"
#include "prefill.cu"
#include "batch.cu"
#include "api.cu"
#include "api_model.cu"
#include "api_ops.cu"
#include "api_noalloc.cu"
#include "tokenizer.cu"
