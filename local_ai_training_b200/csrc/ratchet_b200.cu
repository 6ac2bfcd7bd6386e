// ratchet_b200.cu — the single compilation unit of libratchet_b200.so (sm_100a).  The kernels share
// one device status word, so all sources are compiled together instead of with -rdc.
#include "rt_api.cuh"
#include "rt_rowops.cuh"
#include "rt_gemm.cuh"
#include "rt_loss.cuh"
