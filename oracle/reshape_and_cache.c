/*
 * ORACLE — test infrastructure only.  Not part of the product: nothing in the
 * tecoops library links, loads or calls this file.  Only tests/, the smoke
 * check in __graft_entry__.py and the CPU-baseline leg of bench.py use it, as
 * the checker / the timed reference CPU path.
 *
 * C restatement of the reference's CPU golden for reshape_and_cache:
 * test/zoo/teco/reshape_and_cache/reshape_and_cache.cpp:136-147 (cpuCompute),
 * the same loop the SDAA kernel runs
 * (teco/ual/kernel/reshape_and_cache/reshape_and_cache_fp16.scpp:70-95):
 *
 *   for t in tokens: slot = slot_mapping[t]; if slot < 0: skip
 *     blk = slot / bs; off = slot % bs
 *     for h: key_cache[blk][h][off][:] = key[t][h][:]; same for value
 *
 * Elements are moved as raw 16-bit words (fp16 / bf16 alike), so the result is
 * bit-exact.  Two deliberate differences, both matching the product: offsets are
 * 64-bit (the reference's int offsets overflow past 2^31 elements) and slots
 * >= num_blocks*block_size are skipped (the reference writes out of bounds).
 * `threads` > 1 splits the token loop over OpenMP-free pthreads for the timed
 * CPU baseline; the result does not depend on it when slots are distinct.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    const uint16_t *key, *value;
    const int64_t *slot;
    uint16_t *kc, *vc;
    int64_t t0, t1;
    int H, D, NB, BS;
} rc_job;

static void rc_range(const rc_job *j) {
    const int64_t H = j->H, D = j->D, BS = j->BS;
    const int64_t nslots = (int64_t)j->NB * BS;
    for (int64_t t = j->t0; t < j->t1; ++t) {
        const int64_t slot = j->slot[t];
        if (slot < 0 || slot >= nslots) continue;
        const int64_t blk = slot / BS;
        const int64_t off = slot % BS;
        for (int64_t h = 0; h < H; ++h) {
            const int64_t src = t * H * D + h * D;
            const int64_t dst = blk * H * BS * D + h * BS * D + off * D;
            memcpy(j->kc + dst, j->key + src, (size_t)D * sizeof(uint16_t));
            memcpy(j->vc + dst, j->value + src, (size_t)D * sizeof(uint16_t));
        }
    }
}

static void *rc_thread(void *arg) {
    rc_range((const rc_job *)arg);
    return 0;
}

int oracle_reshape_and_cache(const uint16_t *key, const uint16_t *value, const int64_t *slot,
                             uint16_t *key_cache, uint16_t *value_cache, int64_t num_tokens,
                             int num_kv_heads, int head_size, int num_blocks, int block_size,
                             int threads) {
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    rc_job jobs[64];
    pthread_t tid[64];
    const int64_t per = (num_tokens + threads - 1) / threads;
    for (int i = 0; i < threads; ++i) {
        rc_job j = {key, value, slot, key_cache, value_cache, i * per,
                    (i + 1) * per < num_tokens ? (i + 1) * per : num_tokens,
                    num_kv_heads, head_size, num_blocks, block_size};
        jobs[i] = j;
    }
    if (threads == 1) {
        rc_range(&jobs[0]);
        return 0;
    }
    for (int i = 0; i < threads; ++i) {
        if (jobs[i].t0 >= jobs[i].t1) continue;
        if (pthread_create(&tid[i], 0, rc_thread, &jobs[i]) != 0) {
            rc_range(&jobs[i]);
            jobs[i].t0 = jobs[i].t1;   /* mark done */
            continue;
        }
    }
    for (int i = 0; i < threads; ++i)
        if (jobs[i].t0 < jobs[i].t1) pthread_join(tid[i], 0);
    return 0;
}
