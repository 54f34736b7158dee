/*
 * bs_oracle.h -- CPU oracle for the BigSmall bf16 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (bigsmall_b200/, the
 * C-ABI library) may link, import or call this code.  It is used by tests/
 * as the parity checker, by __graft_entry__.smoke() as the checker, and by
 * bench.py's cpu_baseline / --impl reference legs as the timed CPU port of
 * the reference's own CPU decoders.
 *
 * What it restates (reference paths are relative to the BigSmall project):
 *   - bigsmall/codecs/rans.py            quantise_frequencies, encode_stream,
 *                                        decode_stream (zero-pad quirk kept)
 *   - bigsmall/codecs/bf16_parallel.py   bf16_parallel_v1 "PAR1" encode/decode
 *   - bigsmall/codecs/single_kernel.py   bf16_se_single_kernel encode/decode
 *   - bigsmall/codecs/bf16_tans.py +
 *     bigsmall/codecs/numba_rans.py      bf16_se_tans encode/decode
 * and the CPU reference encoder/decoder of this project's own chunked
 * format bf16_exp_chunked_v1 (no reference counterpart; its parity anchor
 * is the md5 of the raw tensor bytes, as bigsmall/verify.py:44-51 does).
 *
 * Return codes: >= 0 success (byte counts for encoders), < 0 error.
 */
#ifndef BS_ORACLE_H
#define BS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BSO_OK            0
#define BSO_E_ARG        -1
#define BSO_E_MAGIC      -2
#define BSO_E_COUNT      -3
#define BSO_E_TRUNC      -4
#define BSO_E_PREC       -5
#define BSO_E_CAP        -6
#define BSO_E_CORRUPT    -7
#define BSO_E_NOMEM      -8

/* ---- rans.py ------------------------------------------------------------ */
int bso_quantise_ref(const int64_t *counts, int alphabet, uint32_t M,
                     uint32_t *freqs);
int64_t bso_rans_encode(const int32_t *syms, int64_t n, const uint32_t *freqs,
                        int alphabet, uint32_t M, uint8_t *out, int64_t cap);
int bso_rans_decode(const uint8_t *data, int64_t len, int64_t n,
                    const uint32_t *freqs, int alphabet, uint32_t M,
                    uint32_t *out);

/* ---- bf16_parallel_v1 --------------------------------------------------- */
int64_t bso_par_bound(int64_t n, int n_streams);
int64_t bso_par_encode(const uint16_t *w, int64_t n, int n_streams,
                       uint8_t *out, int64_t cap);
int bso_par_decode(const uint8_t *blob, int64_t len, int64_t n_weights,
                   uint16_t *out);

/* ---- bf16_se_single_kernel ---------------------------------------------- */
int64_t bso_sk_bound(int64_t n);
int64_t bso_sk_encode(const uint16_t *w, int64_t n, uint8_t *out, int64_t cap);
int bso_sk_decode(const uint8_t *blob, int64_t len, int64_t n_weights,
                  uint16_t *out);
/* Decode `count` independent blobs on `threads` host threads (the timed CPU
 * baseline).  Returns 0 or the first error code. */
int bso_sk_decode_many(const uint8_t *const *blobs, const int64_t *lens,
                       const int64_t *n_weights, uint16_t *const *outs,
                       int count, int threads);

/* ---- bf16_se_tans ------------------------------------------------------- */
int64_t bso_tans_bound(int64_t n);
int64_t bso_tans_encode(const uint16_t *w, int64_t n, uint8_t *out,
                        int64_t cap);
int bso_tans_decode(const uint8_t *blob, int64_t len, int64_t n_weights,
                    uint16_t *out);

/* ---- bf16_exp_chunked_v1 (this project's format) ------------------------ */
int64_t bso_xc_bound(int64_t n, uint32_t chunk_elems);
int64_t bso_xc_encode(const uint16_t *w, int64_t n, int coder, int prec,
                      uint32_t chunk_elems, uint8_t *out, int64_t cap);
/* chunk_elems values per chunk in `groups` state groups (format version 2
 * when groups > 1; groups == 1 is bso_xc_encode). */
int64_t bso_xc_encode_groups(const uint16_t *w, int64_t n, int coder, int prec,
                             uint32_t chunk_elems, uint32_t groups, uint8_t *out, int64_t cap);
int bso_xc_decode(const uint8_t *blob, int64_t len, int64_t n_weights,
                  uint16_t *out);
/* Quantised exponent frequencies the format uses (for tests). */
int bso_xc_quantise(const int64_t *counts, int prec, uint16_t *freqs);
int bso_tans_decode_many(const uint8_t *const *blobs, const int64_t *lens,
                         const int64_t *n_weights, uint16_t *const *outs, int count, int threads);
int bso_xc_decode_many(const uint8_t *const *blobs, const int64_t *lens,
                       const int64_t *n_weights, uint16_t *const *outs,
                       int count, int threads);
int bso_par_decode_many(const uint8_t *const *blobs, const int64_t *lens,
                        const int64_t *n_weights, uint16_t *const *outs,
                        int count, int threads);

#ifdef __cplusplus
}
#endif
#endif
