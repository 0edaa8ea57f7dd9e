/*
 * ref64.h - float64 CPU reference of the attention forward. TEST INFRASTRUCTURE ONLY: linked by the
 * torch-free harness under tests/harness, never by the library.
 *
 * Restates b4batunde/Phantom-A100 sim/harness.cu:40-64 (its reference()): for every (bh, row),
 * s_j = (q_row . k_j) / sqrt(d) in double, keys after the row masked when causal, p_j = exp(s_j - max),
 * o = sum_j p_j v_j / sum_j p_j.
 */
#ifndef PHANTOM_ORACLE_REF64_H_
#define PHANTOM_ORACLE_REF64_H_

#ifdef __cplusplus
extern "C" {
#endif

/* q, k, v: (BH, N, d) row-major float values; o: (BH, N, d) double output. */
void phantom_ref64_attention(const float* q, const float* k, const float* v, double* o, int BH, int N, int d,
                             int causal);

#ifdef __cplusplus
}
#endif

#endif /* PHANTOM_ORACLE_REF64_H_ */
