// Single translation unit of libmirai_b200.so: the device error word in
// capi.cu is referenced by every kernel, so all parts compile together.
#include "capi.cu"
#include "routing.cu"
#include "plan_static.cu"
#include "grouped_gemm.cu"
#include "quantize.cu"
#include "lora.cu"
#include "exchange.cu"
#include "rotate.cu"
