/* Test infrastructure: the C interface of the CPU restatement in oracle.cpp.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it. */
#ifndef EAGLE_B200_ORACLE_H
#define EAGLE_B200_ORACLE_H
#include <stdint.h>

/* element types and operators: the codes of the reduce seam */
#define ORACLE_F32 0
#define ORACLE_F64 1
#define ORACLE_I32 2
#define ORACLE_I64 3
#define ORACLE_U8 4
#define ORACLE_OP_SUM 0
#define ORACLE_OP_MAX 1
#define ORACLE_OP_ALL 2
#define ORACLE_OP_MIN 3
#define ORACLE_MASK_IS_DROP 1u

#ifdef __cplusplus
extern "C" {
#endif
int oracle_threads(int threads);
int oracle_reduce(const void* in, int64_t n, int64_t cols, int dtype, int op, const void* comp_in, void* out,
    int pair_out);
int oracle_reduce_fixed(const double* in, int64_t n, int64_t cols, const double* comp_in, double* out);
void oracle_ladder(int64_t n, int ER, int G, double* x, long long* units);
int64_t oracle_leaf_partials_f64(const double* x, int64_t n, double* hc);
void oracle_pairwise_f64(const double* hc, int64_t m, double* root_hc);
double oracle_partial_value_f64(double h, double c);
int oracle_compact(const uint8_t* mask, int64_t n, uint32_t flags, int32_t* index_map, uint32_t* count,
    uint32_t span, float theta, uint32_t* live32, uint32_t* fire);
uint32_t oracle_mask_count(const uint8_t* mask, int64_t n);
int64_t oracle_band_k(double rate, int64_t newly, int64_t live, int64_t k, int64_t k_max, int64_t k_min);
void oracle_policy_step(uint32_t finished, uint32_t total, int64_t* cells, int64_t* word, uint32_t* go,
    int64_t* hist, int64_t k_min, int64_t k_max, int iK, int iFin, int iDone, int iCap, int iR, int iMapped,
    int scale);
int oracle_oscillator_run(int64_t n, const double* omega, const double* t_end, double t_end_uniform, double dt,
    double* x, double* v, double* t, uint8_t* term, int32_t* steps_out, int64_t max_steps, int fused,
    int64_t tile, int64_t* stats);
void oracle_philox4x32_10(const uint32_t counter[4], uint64_t seed, uint32_t out[4]);
int oracle_gambler_run(int64_t n, int32_t* pos, int64_t* time, uint8_t* term, int64_t id_base, uint64_t seed,
    int64_t max_steps, int64_t* stats);
double oracle_det_pow(double r, double e);
/* one RKF7(8) attempt's scheme for Lorenz-63: 8th-order state, error vector, mixed max-norm ratio */
void oracle_lorenz_stages(const double s0[3], double step, double rho, double sigma, double beta, double rtol,
    double atol, double s8[3], double err[3], double* ratio);
int oracle_lorenz_run(int64_t n, const double* rho, double sigma, double beta, double t_final, double rtol,
    double atol, double* x, double* y, double* z, double* t, double* h, uint32_t* n_acc, uint32_t* n_rej,
    uint8_t* term, int64_t max_steps, int64_t* stats);
void oracle_corpus_f64(int64_t n, uint64_t seed, double* out);
void oracle_corpus_f32(int64_t n, uint64_t seed, float* out);
double oracle_fixture_f64(int64_t n, double kappa, double* x, double* reached);
double oracle_fixture_f32(int64_t n, double kappa, float* x, double* reached);
#ifdef __cplusplus
}
#endif
#endif
