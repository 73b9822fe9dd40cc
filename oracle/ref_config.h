/*
 * ref_config.h -- forced-include configuration for compiling the qma
 * reference sources in place as a CPU oracle (TEST INFRASTRUCTURE).
 *
 * qma.h hard-codes N_VOCAB = 248320 (qma.h:33) and the LM head always uses
 * N_VOCAB rows (nn.c:2283-2286).  The synthetic models here use the
 * qwen35moe vocabulary of 151936, so after qma.h has been read once (its
 * include guard makes later includes no-ops) N_VOCAB is redefined for the
 * rest of every translation unit.  The qma_t struct keeps its original
 * array sizes, so every TU still agrees on its layout.
 */
#ifndef QMA_REF_CONFIG_H
#define QMA_REF_CONFIG_H
#include "qma.h"
#undef N_VOCAB
#ifndef QMA_REF_N_VOCAB
#define QMA_REF_N_VOCAB 151936
#endif
#define N_VOCAB QMA_REF_N_VOCAB
#endif
