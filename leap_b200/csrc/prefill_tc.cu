// prefill_tc.cu — tensor-core (tcgen05, 3xTF32) causal prefill attention.
#include "common.cuh"
#include "ctx.h"

namespace leap {

int launch_prefill_tc(leap_ctx *c, const float *qrot, const float *kc, const float *vc,
                      float *out, int pos0, int n_tok) {
    (void)c; (void)qrot; (void)kc; (void)vc; (void)out; (void)pos0; (void)n_tok;
    set_error("tensor-core prefill not built for this shape");
    return LEAP_ERR_INVALID;
}

}  // namespace leap
