// Entry points whose kernels are not built yet: they report
// MM4_ERR_UNSUPPORTED so the ABI is complete and callers fail loudly.
#include "mm4_internal.h"

using namespace mm4;

extern "C" {

mm4_status mm4_attention_plan_create(mm4_attention_plan** plan, const mm4_attention_desc*) {
  if (plan) *plan = nullptr;
  return fail(MM4_ERR_UNSUPPORTED, "attention is not built yet");
}
void mm4_attention_plan_destroy(mm4_attention_plan*) {}
const char* mm4_attention_plan_kernel_name(const mm4_attention_plan*) { return ""; }
mm4_status mm4_attention_fwd(const mm4_attention_plan*, const void*, const void*, const void*, void*, mm4_stream_t,
                             int) {
  return fail(MM4_ERR_UNSUPPORTED, "attention is not built yet");
}
}  // extern "C"
