// Single translation unit for libapa_kernels.so: the kernels share the
// device status word (apa::g_status), so they are compiled together rather
// than as relocatable device code.
#include "cast.cu"
#include "gemm.cu"
#include "cast_tma.cu"
#include "ladder.cu"
#include "noalloc.cu"
#include "forensic.cu"
#include "adamw.cu"
#include "dp_nvls.cu"
