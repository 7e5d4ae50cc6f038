// Single translation unit of libjakal_b200.so: the device error word and every
// kernel live in one module, so no relocatable device code is needed.
#include "jk_host.cu"
#include "jk_project.cu"
#include "jk_topk.cu"
#include "jk_window.cu"
#include "jk_split.cu"
#include "jk_noalloc.cu"
