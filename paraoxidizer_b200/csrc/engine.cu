// engine.cu -- decode-step state owned by a context (paged KV cache, model, tensor parallel).
#include "api_internal.h"

namespace pox {
void destroy_ctx_extras(pox_cuda_ctx* ctx) { (void)ctx; }
}  // namespace pox
