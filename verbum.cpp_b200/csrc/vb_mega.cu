// vb_mega.cu -- persistent fused decode step (one launch per token).
// Placeholder until the fused kernel lands: reports "unsupported", which makes
// the engine fall back to the per-op graph path.
#include "vb_engine.cuh"

namespace vb {

vb_status mega_prepare(vb_engine*) {
    return fail(VB_ERR_UNSUPPORTED, "fused step not built");
}
vb_status mega_enqueue_step(vb_engine*, cudaStream_t) {
    return fail(VB_ERR_UNSUPPORTED, "fused step not built");
}
void mega_release(vb_engine* e) { e->mega = nullptr; }

}  // namespace vb
