// Tensor-core split-KV decode for f16 / q8 caches (filled in by the tcgen05/mma kernels).
#include "attn.h"

namespace bg {
int launch_attn_tc(const AttnArgs &, cudaStream_t) { return BG_EUNSUPPORTED; }
}  // namespace bg
