// On-chip resident Sinkhorn solvers: placeholder until the resident kernels
// land; every shape currently takes the streaming path.
#include "internal.h"
#include "sinkhorn.h"

namespace dotb {

bool sk_resident_supported(int64_t, int64_t) { return false; }
size_t sk_resident_fwd_ws(int64_t, int64_t, int64_t, bool) { return 0; }
int sk_resident_fwd(const SkFwdArgs&, void*, cudaStream_t) { return fail(DOT_ERR_UNSUPPORTED, "resident"); }
size_t sk_resident_bwd_ws(int64_t, int64_t, int64_t) { return 0; }
int sk_resident_bwd(const SkBwdArgs&, void*, cudaStream_t) { return fail(DOT_ERR_UNSUPPORTED, "resident"); }

}  // namespace dotb
