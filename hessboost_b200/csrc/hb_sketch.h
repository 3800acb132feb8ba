// Device quantile sketch and binning (hb_sketch.cu), for the engine's upload
// of raw matrices (hb_engine_upload_dense / hb_engine_upload_csr).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "../../include/hb_backend.h"

namespace hb {

// Cuts of a dense row-major f32 matrix (NaN missing) already on the device:
// the reference's HistCuts::from_dmatrix (src/data/quantile.rs:65) with
// unit weights. `fo` gets n_cols + 1 offsets, `cuts` the concatenated cut
// values. HB_REFUSED (with `why`) for inputs the device sketch does not
// take: a feature with 2^24 or more present values, max_bin above 256, or
// more than 2^32 - 1 present cells in all.
hb_status sketch_dense_cuts(int device, const float* d_x, uint64_t n_rows, uint32_t n_cols,
                            uint32_t max_bin, cudaStream_t s, std::vector<uint32_t>& fo,
                            std::vector<float>& cuts, std::string& why);

// Feature-major one-byte local bins and the missing bitmap of a dense
// device matrix (GHistIndex::from_dmatrix, src/data/ghist.rs:213), from
// device cuts. `d_missing` may be NULL; `d_any_missing` (one int, set to 1
// when a cell is missing) is zeroed here first.
cudaError_t bin_dense_device(const float* d_x, uint64_t n_rows, uint32_t n_cols,
                             const uint32_t* d_fo, const float* d_cuts, uint8_t* d_columns,
                             uint64_t* d_missing, int* d_any_missing, cudaStream_t s);

// Cuts of a CSR matrix already on the device (DMatrix::from_csr,
// src/data/dmatrix.rs:459; the sparse branch of quantile.rs:199).
// HB_INVALID_ARGUMENT for offsets that do not start at 0 or descend, a column
// out of range or a non-finite stored value; HB_REFUSED for a row whose
// column indices are not strictly ascending (the host path sorts those), or
// the limits of sketch_dense_cuts.
hb_status sketch_csr_cuts(int device, const uint64_t* d_indptr, const uint32_t* d_indices,
                          const float* d_values, uint64_t n_rows, uint32_t n_cols, uint64_t nnz,
                          uint32_t max_bin, cudaStream_t s, std::vector<uint32_t>& fo,
                          std::vector<float>& cuts, std::string& why);

// Every stored entry's global bin (ascending within a row, because a row's
// columns ascend), and *any_short = 1 when some row lacks a feature.
cudaError_t bin_csr_device(const uint64_t* d_indptr, const uint32_t* d_indices,
                           const float* d_values, uint64_t n_rows, uint32_t n_cols, uint64_t nnz,
                           const uint32_t* d_fo, const float* d_cuts, uint32_t* d_row_bins,
                           int* d_any_short, cudaStream_t s);

}  // namespace hb
