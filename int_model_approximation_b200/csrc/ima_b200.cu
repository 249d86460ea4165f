// Single translation unit of libima_b200.so (the device status word in
// ima_common.cuh is defined once here).
#include "runtime.cu"
#include "quantize.cu"
#include "hawkeye.cu"
#include "freivalds.cu"
#include "int_gemm.cu"
#include "class_counts.cu"
#include "class_count_engine.cu"
