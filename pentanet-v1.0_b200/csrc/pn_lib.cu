// pn_lib.cu -- single translation unit of libpentanet_b200.so.
//
// The kernel files share one device status word (pn::g_device_status); building
// them as one unit keeps that a plain __device__ variable without relocatable
// device code.
#include <cstdarg>

#include "pn_pack.cu"
#include "pn_act.cu"
#include "pn_norm.cu"
#include "pn_dqmm.cu"
#include "pn_simt.cu"
#include "pn_gemv.cu"
#include "pn_capi.cu"
#include "pn_static_ws.cu"
#include "pn_peer.cu"
#include "pn_i8w.cu"
#include "pn_ternary2.cu"
