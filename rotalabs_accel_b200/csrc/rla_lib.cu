// The whole library as one translation unit (no relocatable device code is
// needed for the shared device-side error word).
#include "rla_misc.cu"
#include "rla_skinny.cu"
#include "rla_stream.cu"
#include "rla_tc.cu"
#include "rla_capi.cu"
#include "rla_noalloc.cu"
#include "rla_peer.cu"
#include "rla_xchg.cu"
