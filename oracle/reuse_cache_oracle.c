/*
 * C restatement of the reference's reuse-cache known-answer tests.
 *
 * TEST INFRASTRUCTURE ONLY: loaded with ctypes by tests/ (and by the smoke
 * check) as the checker.  The shadowkv_b200 library never links or calls it.
 *
 * What is restated (reference = WilliamBy/ShadowKV):
 *
 *  - skv_kat_keys: the key generator of kernels/test_cached_gather_copy.cu:
 *    220-282 -- srand(seed); per block, map_size distinct keys
 *    rand() % cpu_chunks, sorted ascending; then fake_hit_cnt "hits" that
 *    pick distinct slots rand() % map_size of the sorted keys, and misses
 *    rand() % cpu_chunks not seen among the block's keys or earlier
 *    reorders.  With seed 12345, 192 blocks, map 256, 16384 chunks and 154
 *    hits this reproduces the reference test's keys exactly (glibc rand()).
 *  - skv_kat_keys_nohit: the generator of kernels/test_gather_copy.cu:
 *    123-167 (FAKE_HIT_CNT = 0 path; that test seeds with time(NULL), a
 *    fixed seed is used here).
 *  - skv_golden_reorder: check_reorder_keys_and_mixed_offsets,
 *    kernels/test_cached_gather_copy.cu:70-156 (std::map lookup, hit keys
 *    and hit offsets each sorted ascending, misses sorted and appended with
 *    offset = key).
 *  - skv_golden_cached_copy: check_cached_copy,
 *    kernels/test_cached_gather_copy.cu:158-216 (slot i < cnt copies 2 KiB
 *    from the device buffer at offsets[i], otherwise from host V).
 *  - skv_golden_gather_copy: check_cached_copy of
 *    kernels/test_gather_copy.cu:67-116 (slot i copies host chunk keys[i]).
 *  - skv_glibc_rand_check: first values of rand() after srand(seed), so a
 *    test can confirm the C library matches glibc's generator.
 *
 * Build: see oracle/build_oracle.py (gcc -O2 -shared -fPIC).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static int cmp_i64(const void *a, const void *b)
{
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

static int cmp_i32(const void *a, const void *b)
{
    int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
    return (x > y) - (x < y);
}

int skv_glibc_rand_check(unsigned seed, int n, int *out)
{
    srand(seed);
    for (int i = 0; i < n; ++i)
        out[i] = rand();
    return 0;
}

/* keys/query: [block_num * map_size] int64 */
int skv_kat_keys(int block_num, int map_size, int cpu_chunks, int fake_hit_cnt, unsigned seed,
                 int64_t *keys, int64_t *query)
{
    char *prev_keys = (char *)malloc((size_t)cpu_chunks);
    char *prev_reorders = (char *)malloc((size_t)cpu_chunks);
    char *prev_hits = (char *)malloc((size_t)map_size);
    if (!prev_keys || !prev_reorders || !prev_hits)
        return -1;
    srand(seed);
    for (int k = 0; k < block_num; ++k) {
        memset(prev_keys, 0, (size_t)cpu_chunks);
        memset(prev_reorders, 0, (size_t)cpu_chunks);
        memset(prev_hits, 0, (size_t)map_size);
        for (int i = 0; i < map_size; ++i) {
            int key;
            do {
                key = rand() % cpu_chunks;
            } while (prev_keys[key]);
            prev_keys[key] = 1;
            keys[(int64_t)k * map_size + i] = key;
        }
        qsort(keys + (int64_t)k * map_size, (size_t)map_size, sizeof(int64_t), cmp_i64);
        for (int i = 0; i < map_size; ++i) {
            int64_t idx = (int64_t)k * map_size + i;
            if (i < fake_hit_cnt) {
                int hr;
                do {
                    hr = rand() % map_size;
                } while (prev_hits[hr]);
                prev_hits[hr] = 1;
                query[idx] = keys[(int64_t)k * map_size + hr];
            } else {
                int r;
                do {
                    r = rand() % cpu_chunks;
                } while (prev_reorders[r] || prev_keys[r]);
                query[idx] = r;
            }
            prev_reorders[query[idx]] = 1;
        }
    }
    free(prev_keys);
    free(prev_reorders);
    free(prev_hits);
    return 0;
}

int skv_kat_keys_nohit(int block_num, int map_size, int cpu_chunks, unsigned seed,
                       int64_t *keys, int64_t *query)
{
    char *prev_keys = (char *)malloc((size_t)cpu_chunks);
    char *prev_reorders = (char *)malloc((size_t)cpu_chunks);
    if (!prev_keys || !prev_reorders)
        return -1;
    srand(seed);
    for (int k = 0; k < block_num; ++k) {
        memset(prev_keys, 0, (size_t)cpu_chunks);
        memset(prev_reorders, 0, (size_t)cpu_chunks);
        for (int i = 0; i < map_size; ++i) {
            int key;
            do {
                key = rand() % cpu_chunks;
            } while (prev_keys[key]);
            prev_keys[key] = 1;
            keys[(int64_t)k * map_size + i] = key;
        }
        for (int i = 0; i < map_size; ++i) {
            int64_t idx = (int64_t)k * map_size + i;
            (void)(rand() % 256); /* the "hit" draw; never < FAKE_HIT_CNT = 0 */
            int r;
            do {
                r = rand() % cpu_chunks;
            } while (prev_reorders[r]);
            query[idx] = r;
            prev_reorders[r] = 1;
        }
    }
    free(prev_keys);
    free(prev_reorders);
    return 0;
}

typedef struct {
    int64_t key;
    int slot;
} kv_t;

static int cmp_kv(const void *a, const void *b)
{
    const kv_t *x = (const kv_t *)a, *y = (const kv_t *)b;
    if (x->key != y->key)
        return (x->key > y->key) - (x->key < y->key);
    return (x->slot > y->slot) - (x->slot < y->slot);
}

/* out_keys int64, out_offsets int32, cnts int32 (hit count per block) */
int skv_golden_reorder(int block_num, int map_size, const int64_t *orig, const int64_t *query,
                       int64_t *out_keys, int32_t *out_offsets, int32_t *cnts)
{
    kv_t *lut = (kv_t *)malloc(sizeof(kv_t) * (size_t)map_size);
    int64_t *miss = (int64_t *)malloc(sizeof(int64_t) * (size_t)map_size);
    if (!lut || !miss)
        return -1;
    for (int k = 0; k < block_num; ++k) {
        const int64_t *o = orig + (int64_t)k * map_size;
        const int64_t *q = query + (int64_t)k * map_size;
        int64_t *rk = out_keys + (int64_t)k * map_size;
        int32_t *ro = out_offsets + (int64_t)k * map_size;
        for (int i = 0; i < map_size; ++i) {
            lut[i].key = o[i];
            lut[i].slot = i;
        }
        /* std::map::insert keeps the first value for a repeated key: after
         * sorting by (key, slot) the first entry of a run is that value. */
        qsort(lut, (size_t)map_size, sizeof(kv_t), cmp_kv);
        int idw = 0, nmiss = 0;
        for (int i = 0; i < map_size; ++i) {
            int lo = 0, hi = map_size - 1, found = -1;
            while (lo <= hi) {
                int mid = (lo + hi) / 2;
                if (lut[mid].key < q[i])
                    lo = mid + 1;
                else {
                    if (lut[mid].key == q[i])
                        found = mid;
                    hi = mid - 1;
                }
            }
            if (found >= 0) {
                rk[idw] = q[i];
                ro[idw] = lut[found].slot;
                idw++;
            } else {
                miss[nmiss++] = q[i];
            }
        }
        qsort(rk, (size_t)idw, sizeof(int64_t), cmp_i64);
        qsort(ro, (size_t)idw, sizeof(int32_t), cmp_i32);
        qsort(miss, (size_t)nmiss, sizeof(int64_t), cmp_i64);
        cnts[k] = idw;
        for (int i = 0; i < nmiss; ++i) {
            rk[idw] = miss[i];
            ro[idw] = (int32_t)miss[i];
            idw++;
        }
    }
    free(lut);
    free(miss);
    return 0;
}

/*
 * host_v:  [block_num][cpu_v_length] bf16 (2-byte units)
 * dev_v:   [block_num][gpu_v_length] bf16 -- the device buffer BEFORE the copy
 * golden:  [block_num][map_size][1024] bf16 -- slot-major result
 */
int skv_golden_cached_copy(int block_num, int map_size, int64_t cpu_v_length, int64_t gpu_v_length,
                           const uint16_t *host_v, const uint16_t *dev_v, const int32_t *offsets,
                           const int32_t *cnts, uint16_t *golden)
{
    for (int64_t k = 0; k < block_num; ++k) {
        for (int64_t i = 0; i < map_size; ++i) {
            int64_t idx = k * map_size + i;
            const uint16_t *src;
            if (i < cnts[k])
                src = dev_v + k * gpu_v_length + (int64_t)offsets[idx] * 1024;
            else
                src = host_v + k * cpu_v_length + (int64_t)offsets[idx] * 1024;
            memcpy(golden + idx * 1024, src, 2048);
        }
    }
    return 0;
}

int skv_golden_gather_copy(int block_num, int map_size, int64_t cpu_v_length,
                           const uint16_t *host_v, const int64_t *keys, uint16_t *golden)
{
    for (int64_t k = 0; k < block_num; ++k) {
        for (int64_t i = 0; i < map_size; ++i) {
            int64_t idx = k * map_size + i;
            memcpy(golden + idx * 1024, host_v + k * cpu_v_length + keys[idx] * 1024, 2048);
        }
    }
    return 0;
}
