/*
 * CPU oracle for the exact k-NN hot path of mlxVS (test infrastructure only).
 *
 * This is a plain-C restatement of the reference algorithm, used as the
 * checker by tests/, by __graft_entry__.smoke() and by bench.py's CPU
 * baseline leg.  The product (mlxvs_b200) never links or calls it.
 *
 * Parity status: the reference (MLX + Metal, macOS only) cannot be built or
 * run on Linux, so this oracle is pinned against the reference's own
 * known-answer tests, restated in tests/test_oracle.py:
 *   - ties KAT            tests/test_knn.cpp:158-192
 *   - Hamming tiny KAT    python/tests/test_cuvs.py:844-849
 *   - n < k padding       python/tests/test_mlxvs.py:63-69
 *   - recall / rtol sweep tests/test_knn.cpp:56-113, python/tests/test_mlxvs.py:30-48
 *   - Hamming vs popcount tests/test_ivf.cpp:252-311
 *
 * Ordering contract (src/kernels.h:14-23): a candidate (score s, id i) comes
 * before (s', i') when s > s', or s == s' and (uint32)i < (uint32)i'.  Both
 * are folded into one 64-bit key, larger = better:
 *   key = (order_bits(s) << 32) | (uint32)~i
 * where order_bits is the sign-flip map of src/kernels.h:16-19.
 */
#ifndef MLXVS_ORACLE_H
#define MLXVS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_IP = 0, ORACLE_L2 = 1, ORACLE_COSINE = 2 };

/* 0 = ok, 1 = invalid argument (k outside [1,256], d < 1, n/nq < 0). */
int oracle_brute_force_knn(const float* base, int64_t n, const float* queries,
                           int64_t nq, int32_t d, int32_t k, int32_t metric,
                           int32_t* ids, float* distances, int32_t threads);

int oracle_hamming_knn(const uint8_t* rows, int64_t n, const uint8_t* queries,
                       int64_t nq, int32_t bytes, int32_t k, int32_t* ids,
                       float* distances, int32_t threads);

/* Best k of L sorted-or-unsorted candidate lists per query.  lists is laid
 * out [L][nq][k] of 64-bit keys (0 = empty slot); out is [nq][k], best
 * first, 0-padded. */
void oracle_merge_keys(const uint64_t* lists, int32_t L, int64_t nq, int32_t k,
                       uint64_t* out);

uint64_t oracle_key(float score, int32_t id);

/* Raw (pre-distance) scores of the k best per query: L2 scores are
 * 2 q.b - |b|^2 (src/knn.cpp:111-116), others the dot / cosine.  ids as in
 * oracle_brute_force_knn, id_offset added.  Used to check the sharded path. */
int oracle_knn_keys(const float* base, int64_t n, const float* queries,
                    int64_t nq, int32_t d, int32_t k, int32_t metric,
                    int64_t id_offset, uint64_t* keys, int32_t threads);

#ifdef __cplusplus
}
#endif

#endif
