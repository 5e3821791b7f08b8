// tma_host.h -- host-side encoding of the 2-D tensor maps the kernels copy
// packed weight rows with (the driver's cuTensorMapEncodeTiled).
#pragma once

#include <cstdint>

#include <cuda.h>

namespace clq {

// ROWS rows of ROW_BYTES bytes at BASE (16-byte aligned), read as boxes of
// BOX_ROWS rows x BOX bytes (BOX a multiple of 16, at most 256; rows past the
// end read as zeros).  False when the driver entry point is missing or the
// geometry is not allowed.
bool encode_rows(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box, int box_rows);

}  // namespace clq
