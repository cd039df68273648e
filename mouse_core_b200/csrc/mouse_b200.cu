// Single translation unit of libmouse_b200.so: the kernels share the device
// status word without relocatable device code.
#include "decode_attention.cu"
#include "kv_append.cu"
#include "elementwise.cu"
#include "train_elementwise.cu"
#include "segment_meta.cu"
#include "varlen_attention.cu"
#include "varlen_backward.cu"
#include "packing.cu"
#include "embed.cu"
#include "td_loss.cu"
#include "capi.cu"
#include "decode_noalloc.cu"
