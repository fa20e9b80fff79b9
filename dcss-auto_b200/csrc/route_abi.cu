// The route-cue task under the reference's learn_* names (libd1_route.so): thin
// forwards to the d1_route_* entry points of route_env.cu.
#include "../../include/d1_route.h"

extern "C" {

int learn_state_bytes(void) { return d1_route_state_bytes(); }
int learn_obs_size(void) { return d1_route_obs_size(); }
int learn_action_size(void) { return d1_route_action_size(); }
int learn_out_size(void) { return d1_route_out_size(); }
int learn_config_bytes(void) { return d1_route_config_bytes(); }

int learn_init(void *state, int n, const D1Config *c, const D1RouteTables *t, uint64_t seed, float *obs, float *mask,
               void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    return d1_route_init(state, n, c, t, seed, obs, mask, nullptr, stream);
}

int learn_step(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions, int limit,
               float *obs, float *mask, float *out, void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    return d1_route_step(state, n, c, t, actions, limit, obs, mask, out, nullptr, nullptr, stream);
}

int learn_step_active(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions,
                      int limit, float *obs, float *mask, float *out, const bool *active, void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    return d1_route_step(state, n, c, t, actions, limit, obs, mask, out, active, nullptr, stream);
}

int learn_heuristic(void *state, int n, const D1Config *c, const D1RouteTables *t, int64_t *actions, void *stream,
                    int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    return d1_route_heuristic(state, n, c, t, actions, stream);
}

}  // extern "C"
