// paged.cu - read lists over a paged KV cache: positions -> physical slots (sm_100a).
//
// Reference (AIwork4me/latent-sparse-attention-rocm, src/lsa_rocm_lab/port/select_fused.py):
// the expansion walk's MAP_SLOTS path (:147-148, :177-199) loads row r's slot-table row
// slot_rows[r] and stores slot_table[slot_row, id] instead of the position id, for the
// walked bucket members and for the window / sink tail alike. Here the mapping is its own
// pass over finished read lists, so every selection arm (flat, fused, batched, tree,
// positional) composes with it; the lists it writes equal the mapped walk's entry for entry.
// Positions outside the table (or a row whose slot row is outside it) map to -1, which the
// read skips.
#include "common.cuh"

namespace lsa {

__global__ void map_slots_kernel(const int32_t* __restrict__ lists, const int32_t* __restrict__ lengths, int64_t R,
                                 int64_t width, const int32_t* __restrict__ table, int64_t table_rows,
                                 int64_t table_cols, int64_t ld_table, const int32_t* __restrict__ slot_rows,
                                 int32_t* __restrict__ out) {
    const int64_t r = blockIdx.y;
    if (r >= R) return;
    int len = lengths[r];
    len = len < 0 ? 0 : (len > width ? (int)width : len);
    const int32_t srow = slot_rows[r];
    const bool row_ok = srow >= 0 && srow < table_rows;
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < width; j += (int64_t)gridDim.x * blockDim.x) {
        int32_t v = -1;
        if (j < len && row_ok) {
            const int32_t id = lists[r * width + j];
            if (id >= 0 && id < table_cols) v = table[(int64_t)srow * ld_table + id];
        }
        out[r * width + j] = v;
    }
}

}  // namespace lsa

extern "C" {

int lsa_map_slots(const int32_t* lists, const int32_t* lengths, int64_t R, int64_t width, const int32_t* slot_table,
                  int64_t table_rows, int64_t table_cols, int64_t ld_table, const int32_t* slot_rows, int32_t* out,
                  cudaStream_t stream) {
    if (R < 0 || width < 0 || table_rows < 0 || table_cols < 0 || ld_table < table_cols) return LSA_ERR_ARG;
    if (R == 0 || width == 0) return LSA_OK;
    if (R > 65535) return LSA_ERR_SIZE;
    dim3 grid((unsigned)((width + 255) / 256 < 16 ? (width + 255) / 256 : 16), (unsigned)R);
    lsa::map_slots_kernel<<<grid, 256, 0, stream>>>(lists, lengths, R, width, slot_table, table_rows, table_cols,
                                                    ld_table, slot_rows, out);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // extern "C"
