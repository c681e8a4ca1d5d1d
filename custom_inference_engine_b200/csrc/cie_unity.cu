// Single translation unit for libcie_attention.so: the device error word
// (cie::g_device_errors) is shared by every kernel without relocatable
// device code.
#include "cie_api.cu"
#include "decode_attention.cu"
#include "decode_noalloc.cu"
#include "kv_update.cu"
#include "lm_head.cu"
#include "rope_kv.cu"
#include "mixed_attention.cu"
