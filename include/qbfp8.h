/*
 * qbfp8.h — C ABI of the BFP8_B weight format and the projection GEMVs that
 * read it, on B200 (sm_100a).  Part of libqcache.so; includes qcache.h for the
 * status codes, qc_stream and qc_last_error().
 *
 * These are the matrix-vector products on either side of the cache path: the
 * combined DeltaNet projection (12352 x 4096), the attention QKV projection
 * (10240 x 4096), the output projections and the FFN, all stored as BFP8_B
 * tiles.  In the reference they run on Tenstorrent cores:
 *   qc_bfp8_gemv        replaces dispatch_gemv        (src/engine.cpp:371-486)
 *   qc_bfp8_gemv_resadd replaces dispatch_gemv_resadd (src/engine.cpp:498-608)
 *   qc_bfp8_gemv_split  replaces dispatch_gemv_split  (src/engine.cpp:619-727)
 *   qc_bfp8_upload      replaces upload_packed_bfp8b_buf (src/engine.cpp:1925-1981)
 *                       for weights read from a type-200 GGUF tensor
 *                       (src/gguf_loader.cpp:151-153)
 *   qc_bfp8_pack_bf16   replaces pack_bf16_as_bfp8b   (src/engine.cpp:1831-1852)
 *
 * Format (GGUF type 200): (M/32)*(K/32) tiles of 1088 bytes, tile (mt, kt) at
 * index mt*(K/32) + kt.  A tile is 4 faces of 16x16 (face 0 rows 0-15 cols
 * 0-15, face 1 rows 0-15 cols 16-31, face 2 rows 16-31 cols 0-15, face 3 rows
 * 16-31 cols 16-31); bytes [0,64) hold one shared exponent per face row
 * (byte f*16 + r), bytes [64,1088) one sign/magnitude byte per element
 * (byte 64 + f*256 + r*16 + c).  Element value =
 * (-1)^(b>>7) * (b & 127) * 2^(exp - 133).
 *
 * Semantics: x is bf16 [batch][K] (row stride K), y bf16 [batch][M] (row
 * stride M); y[b][m] = bf16_rne(sum_k W[m][k] * x[b][k]) with f32
 * accumulation.  resadd: residual[b][m] = bf16_trunc(bf16_rne(Wx) +
 * residual[b][m]), the reference writer's rounding
 * (src/kernels/dataflow/writer_gemv_resadd.cpp).  split: rows < split_m go to
 * y0 [batch][split_m], rows >= split_m to y1 [batch][M - split_m].
 *
 * A matrix object owns its device tiles and the GEMV scratch (split-K partial
 * sums).  Calls on one matrix must not
 * overlap on the GPU (enqueue them on one stream, or serialise the streams);
 * different matrices are independent.  The calls are CUDA-graph capturable.
 * Every call returns QC_OK or an error code; qc_last_error(NULL) describes the
 * last failure of the calling thread.
 */
#ifndef QBFP8_H
#define QBFP8_H

#include "qcache.h"

#ifdef __cplusplus
extern "C" {
#endif

#define QC_BFP8_TILE_BYTES 1088

typedef struct qc_bfp8_matrix qc_bfp8_matrix;

/* Bytes of the packed form of an M x K matrix (M, K multiples of 32). */
int64_t qc_bfp8_packed_bytes(int32_t M, int32_t K);

/* Allocates an M x K matrix (tiles zeroed) and its scratch on `device`. */
int qc_bfp8_create(int device, int32_t M, int32_t K, qc_bfp8_matrix** out);
void qc_bfp8_destroy(qc_bfp8_matrix* m);

/* Device address of the tiles (qc_bfp8_packed_bytes(M, K) bytes).  On the
 * device each tile is kept in a GEMV-friendly permutation of its 1088 bytes;
 * upload/download convert from/to the GGUF layout. */
void* qc_bfp8_tiles(const qc_bfp8_matrix* m);

/* Host packed tiles (GGUF type-200 bytes) -> device, asynchronous on stream;
 * the host buffer must stay valid until the copy completes. */
int qc_bfp8_upload(qc_bfp8_matrix* m, const void* packed_host, qc_stream stream);
/* Device tiles -> host buffer in the GGUF layout, asynchronous on stream
 * (the tiles are permuted back and forth in place around the copy). */
int qc_bfp8_download(qc_bfp8_matrix* m, void* packed_host, qc_stream stream);
/* Packs a row-major bf16 [M][K] device matrix into the tiles on the GPU,
 * byte-identical to the CPU packer of the format. */
int qc_bfp8_pack_bf16(qc_bfp8_matrix* m, const uint16_t* w_dev, qc_stream stream);

int qc_bfp8_gemv(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch, uint16_t* y_dev,
                 qc_stream stream);
int qc_bfp8_gemv_resadd(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch,
                        uint16_t* residual_dev, qc_stream stream);
int qc_bfp8_gemv_split(qc_bfp8_matrix* m, const uint16_t* x_dev, int32_t batch, int32_t split_m,
                       uint16_t* y0_dev, uint16_t* y1_dev, qc_stream stream);

/* Synchronises the device and reports a device-side error of this matrix's
 * kernels (QC_ERR_TIMEOUT from a bounded pipeline wait), then clears it. */
int qc_bfp8_check(qc_bfp8_matrix* m);

#ifdef __cplusplus
}
#endif

#endif /* QBFP8_H */
