/* libd1_route.so -- the route-cue task of include/d1.h ("route") exported under
 * the reference's own names, so that the reference's ctypes wrapper for that
 * task (gpu-d1/scripts/learn_env_ring_multi.py:24-42, which loads one learn.so
 * per variant through library(path)) binds it unchanged. Same argument order
 * and meaning as gpu-d1/src/learn.cu:643-676 built with the route flags; the
 * tables argument is the MULTI_MAP struct (D1RouteTables). There is no host
 * path: gpu == 0 returns D1_ERR_NO_HOST_PATH. State rows are opaque, 13,312
 * bytes (the reference's are 45,288). */
#ifndef D1_ROUTE_H
#define D1_ROUTE_H
#define D1_ROUTE_LIBRARY
#include "d1.h"

#ifdef __cplusplus
extern "C" {
#endif

int learn_state_bytes(void);   /* learn.cu:644 */
int learn_obs_size(void);      /* learn.cu:645: 421 */
int learn_action_size(void);   /* learn.cu:646: 9 */
int learn_out_size(void);      /* learn.cu:647: 8 */
int learn_config_bytes(void);  /* learn.cu:648: 140 */
/* learn.cu:649-660 */
int learn_init(void *state, int n, const D1Config *c, const D1RouteTables *t, uint64_t seed, float *obs, float *mask,
               void *stream, int gpu);
/* learn.cu:661-665 */
int learn_step(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions, int limit,
               float *obs, float *mask, float *out, void *stream, int gpu);
/* learn.cu:666-670 */
int learn_step_active(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions,
                      int limit, float *obs, float *mask, float *out, const bool *active, void *stream, int gpu);
/* learn.cu:671-675 */
int learn_heuristic(void *state, int n, const D1Config *c, const D1RouteTables *t, int64_t *actions, void *stream,
                    int gpu);

#ifdef __cplusplus
}
#endif
#endif
