// bybycuda.cu - the single translation unit of libbybycuda.so (the routes share the device
// error word, so they are compiled together).
#include "abi.cu"
#include "simt.cu"
#include "gemv.cu"
#include "q4asym.cu"
#include "f16gemv.cu"
#include "tc.cu"
#include "tcf16.cu"
#include "vm.cu"
#include "session.cu"
#include "shard.cu"
#include "tune.cu"
#include "ingest.cu"
