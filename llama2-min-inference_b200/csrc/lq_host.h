/* Internal host-side declarations shared by the C and CUDA sources. */
#ifndef LQ_HOST_H
#define LQ_HOST_H

#include <stdint.h>
#include <stddef.h>

#include "../../include/llama2q.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LQ_MAGIC_Q8 0x384C4C51u /* "QLL8", tools/quantize_int8.py:48 */
#define LQ_MAGIC_Q4 0x344C4C51u /* "QLL4", tools/quantize_int4.py:34 */

/* tensor ids, in file order; also the synthetic generator's stream ids */
enum {
    LQ_T_EMB = 0, LQ_T_RMS_ATT, LQ_T_WQ, LQ_T_WK, LQ_T_WV, LQ_T_WO, LQ_T_RMS_FFN,
    LQ_T_W1, LQ_T_W2, LQ_T_W3, LQ_T_RMS_FINAL, LQ_T_WCLS, LQ_NT
};

typedef struct {
    int id;
    int64_t rows, cols;
    int quantized;
} LqTensorDesc;

int lq_tensor_table(const Config* c, LqTensorDesc out[LQ_NT]);
int lq_parse_header(const uint8_t* p, size_t size, Config* cfg, int* kind, int* gs, int* shared,
                    size_t* header_bytes);
int64_t lq_qtensor_bytes(int64_t rows, int64_t cols, int gs, int kind);
void lq_quantize_rows_host(const float* w, int64_t rows, int64_t cols, int gs, int kind,
                           uint8_t* q, float* s);

/* record an error message for lq_last_error() and return code */
int lq_fail(int code, const char* fmt, ...);

#ifdef __cplusplus
}
#endif
#endif
