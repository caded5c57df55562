// Placeholder until the tcgen05 flash attention lands.
#include "kernels.h"
namespace fb {
int launch_attention_tc(const AttnArgs&, void*) { return FB_ERR_UNSUPPORTED; }
}  // namespace fb
