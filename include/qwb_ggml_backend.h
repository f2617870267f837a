/* qwb_ggml_backend.h - the ggml backend built on libqwb.so (libggml-qwb.so).
 *
 * What it replaces.  QuestWend runs its graphs through ggml backends that it loads with
 * ggml_backend_load_all() (core/backend_loader.h:21-24) and schedules with
 * ggml_backend_sched (core/runtime.cpp).  libggml-qwb.so is one more such backend, for
 * B200 (sm_100) devices, implementing the backend interface of ggml-backend-impl.h
 * (interface version 3: buffer type :17-39, buffer :50-79, backend :122-164, device
 * :177-225, registry :231-247).  It computes
 *   GGML_OP_MUL_MAT_ID  on Q4_K / Q6_K / Q8_0 expert tensors      -> qwb_mul_mat_id
 *   GGML_OP_MUL_MAT     on 2-D Q4_K / Q6_K / Q8_0 weights          -> qwb_mul_mat
 *   GGML_OP_GET_ROWS    on Q4_K / Q6_K / Q8_0 / F16 / F32 / I32     -> qwb_get_rows
 * and reports every other compute op unsupported, so the scheduler places those on
 * ggml-cuda or the CPU backend.  Tensors live in the device's buffer type (cudaMalloc'd
 * device memory); a tensor in a buffer marked GGML_BACKEND_BUFFER_USAGE_WEIGHTS (as the
 * model loader marks expert weights, core/model.cpp:244) pulls its MUL_MAT_ID onto this
 * backend.
 *
 * Loading.  Either link the library and call ggml_backend_qwb_reg() +
 * ggml_backend_register(), or leave it beside the other ggml backend libraries and let
 * ggml_backend_load() / ggml_backend_load_all() find it through the two entry points of
 * ggml's dynamic loader below (score 100 when a B200 is visible, 0 otherwise, so hosts
 * without one skip it).
 *
 * ggml_backend_dev_init(dev, params) takes "workspace_mb=N": MUL_MAT_ID scratch reserved
 * when the backend is created (default 256).  graph_compute grows it when a graph needs
 * more, except under CUDA stream capture, where it fails the graph instead of allocating.
 * graph_compute only queues work; ggml_backend_synchronize() waits and prints any
 * out-of-range expert or row ids the kernels met (their outputs are zeroed; the reference
 * CPU backend aborts on such ids). */
#ifndef QWB_GGML_BACKEND_H
#define QWB_GGML_BACKEND_H

#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The registry of the process's B200 devices ("QWB0", "QWB1", ...). */
ggml_backend_reg_t ggml_backend_qwb_reg(void);

/* ggml's dynamic-backend entry points (ggml-backend-impl.h:252-255). */
ggml_backend_reg_t ggml_backend_init(void);
int ggml_backend_score(void);

#ifdef __cplusplus
}
#endif

#endif /* QWB_GGML_BACKEND_H */
