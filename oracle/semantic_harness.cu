// Test infrastructure only: nothing in the product links this file. It is built
// into oracle/_ref/ by `make -C oracle ref` and loaded by tests/ as a checker.
//
// A host-side driver for the rule functions of the reference's semantic-actions
// build (gpu-d1/branches/semantic-actions-v1/src/learn.cu, compiled from its
// sources in place with the flags of that branch's scripts/assets.py). The
// reference's own file is included below, unchanged; the hooks here only build a
// state by hand and call the reference's transition, observe, adjacent_attack,
// visible_awake and monster_detects_player on it, on the host.
//
// Hand-built states follow the shape of the reference's own self-test
// (semantic-actions-v1/src/semantic_tests.cu:3-8): an empty level on map 0 (no
// living monster, every cell in view remembered, all slots free), then monsters
// placed one by one with their discovery slots updated.
#include <cstddef>

#include "learn.cu"

namespace {
enum Field {
    F_HP = 0, F_REGEN, F_PLAYER, F_TICKS, F_KILLED, F_POS, F_ENERGY, F_MHP, F_AWAKE, F_OCC, F_VIEWED, F_SEEN,
    F_FLOOR_SEEN, F_ENEMY_SLOT, F_COUNT
};
}

extern "C" {

int sem_state_bytes() { return (int)sizeof(State); }
int sem_obs_size() { return OBS; }
int sem_out_size() { return OUT; }
int sem_action_size() { return ACTIONS; }
int sem_enemies() { return ENEMIES; }
int sem_required() { return REQUIRED; }

// Byte offset of a State field (enum Field), for reading states from Python.
int sem_offset(int field) {
    switch (field) {
        case F_HP: return (int)offsetof(State, w.hp);
        case F_REGEN: return (int)offsetof(State, w.regen);
        case F_PLAYER: return (int)offsetof(State, player);
        case F_TICKS: return (int)offsetof(State, ticks);
        case F_KILLED: return (int)offsetof(State, killed);
        case F_POS: return (int)offsetof(State, pos);
        case F_ENERGY: return (int)offsetof(State, energy);
        case F_MHP: return (int)offsetof(State, hp);
        case F_AWAKE: return (int)offsetof(State, awake);
        case F_OCC: return (int)offsetof(State, occ);
        case F_VIEWED: return (int)offsetof(State, viewed);
        case F_SEEN: return (int)offsetof(State, seen);
        case F_FLOOR_SEEN: return (int)offsetof(State, floor_seen);
        case F_ENEMY_SLOT: return (int)offsetof(State, enemy_slot);
        default: return -1;
    }
}

// Empty level: the player alone on map 0 at `player` with `hp`, PCG stream
// seeded (mix(seed), 1), ticks `ticks`, every in-view cell remembered.
void sem_empty(State *s, const Config *c, const Tables *t, int player, int hp, int ticks, uint64_t seed) {
    std::memset(s, 0, sizeof(State));
    s->w.rng.seed(mix(seed), 1);
    s->map_id = 0;
    s->player = player;
    s->w.hp = hp;
    s->ticks = ticks;
    for (int p = 0; p < N; p++) {
        s->occ[p] = -1;
        s->frontier_slot[p] = -1;
    }
    for (int j = 0; j < ENEMIES; j++) {
        s->enemy_slot[j] = -1;
        s->energy[j] = -30000;
    }
    reveal(*s, *t);
    update_knowledge(*s, *c, *t);
}

// Monster `id` (kind c.kinds[id % 6] below REQUIRED) at `pos` with `hp`.
void sem_put(State *s, const Config *c, const Tables *t, int id, int pos, int hp, int awake) {
    s->pos[id] = (int16_t)pos;
    s->hp[id] = (int16_t)hp;
    s->occ[pos] = (int16_t)id;
    s->awake[id] = (int16_t)awake;
    update_knowledge(*s, *c, *t);
}

void sem_transition(State *s, const Config *c, const Tables *t, int action, int limit, float *out) {
    transition(*s, *c, *t, action, limit, out);
}

// One physical turn with primitive d (0-7 a step or bump in compass order, 8 a wait).
void sem_primitive(State *s, const Config *c, const Tables *t, int d, int limit, float *out) {
    primitive_transition(*s, *c, *t, d, limit, out);
}

void sem_observe(State *s, const Config *c, const Tables *t, float *obs, float *mask) {
    observe(*s, *c, *t, obs, mask);
}

int sem_adjacent_attack(const State *s, const Config *c, const Tables *t) { return adjacent_attack(*s, *c, *t); }

int sem_visible_awake(const State *s, const Config *c, const Tables *t) { return visible_awake(*s, *c, *t); }

int sem_in_view(const State *s, const Tables *t, int target) { return in_view(*s, *t, target); }

// Whether a sleeping monster standing at `origin` would notice the player.
int sem_detects(const State *s, const Tables *t, int origin) { return monster_detects_player(*s, *t, origin); }

}  // extern "C"
