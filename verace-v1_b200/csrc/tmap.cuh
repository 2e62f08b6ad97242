// Host side of the TMA tensor maps: the driver's cuTensorMapEncodeTiled, resolved once
// through the runtime (the library links no driver import library).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

namespace verace {

// nullptr when the driver does not provide the entry point.
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder();

}  // namespace verace
