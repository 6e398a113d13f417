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
mm4_status mm4_conv2d_plan_create(mm4_conv_plan** plan, const mm4_conv2d_desc*) {
  if (plan) *plan = nullptr;
  return fail(MM4_ERR_UNSUPPORTED, "conv is not built yet");
}
mm4_status mm4_conv3d_plan_create(mm4_conv_plan** plan, const mm4_conv3d_desc*) {
  if (plan) *plan = nullptr;
  return fail(MM4_ERR_UNSUPPORTED, "conv is not built yet");
}
void mm4_conv_plan_destroy(mm4_conv_plan*) {}
const char* mm4_conv_plan_kernel_name(const mm4_conv_plan*) { return ""; }
int64_t mm4_conv_output_elements(const mm4_conv_plan*) { return 0; }
mm4_status mm4_conv_run(const mm4_conv_plan*, const void*, const void*, const void*, void*, mm4_stream_t, int) {
  return fail(MM4_ERR_UNSUPPORTED, "conv is not built yet");
}
mm4_status mm4_permute_weights(int, int, const int32_t*, const void*, void*, mm4_stream_t) {
  return fail(MM4_ERR_UNSUPPORTED, "permute is not built yet");
}

}  // extern "C"
