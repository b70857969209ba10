// tcgen05 symmetric rank-k update (placeholder until the tensor-core kernel lands).
#include "ops.h"

namespace llmc {
llmc_status syrk_tc(llmc_ctx*, const void*, int, int64_t, int64_t, int64_t, float*, int64_t) {
    return LLMC_ERR_UNSUPPORTED;
}
}  // namespace llmc
