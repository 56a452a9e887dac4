// tcgen05 tensor-core path of the repacked GEMM (filled in by the sm_100a kernel).
#include "jkb_internal.h"

namespace jkb {

int gemm_tc_launch(const jkb_repacked_weight *w, const jkb_act_q8 *act, float *out,
                   size_t row_begin, size_t row_end, cudaStream_t st, bool *used) {
    (void)w; (void)act; (void)out; (void)row_begin; (void)row_end; (void)st;
    *used = false;
    return JKB_OK;
}

}  // namespace jkb
