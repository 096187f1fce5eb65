/*
 * runtime.c -- error reporting, stream selection, pointer residency, workspace and
 * synchronisation for the host C layer.
 *
 * The reference's attention and append functions return void with no error channel
 * (kernel/attention.h:11,26,39); here every entry point records failures in a
 * thread-local message read through attn_last_error().
 */
#include <cuda_runtime_api.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "attn_ext.h"
#include "host_internal.h"

static _Thread_local char g_err[512];
static _Thread_local void *g_stream; /* NULL: legacy default stream */

void tyb_set_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int tyb_cuda_ok(int err, const char *what)
{
    if (err == 0) return 1;
    tyb_set_error("%s: %s", what, cudaGetErrorString((cudaError_t)err));
    return 0;
}

const char *attn_last_error(void) { return g_err; }

void attn_clear_error(void) { g_err[0] = '\0'; }

void attn_set_stream(void *stream) { g_stream = stream; }

void *tyb_stream(void) { return g_stream; }

int tyb_is_device_ptr(const void *p)
{
    struct cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError(); /* clear the sticky-free error state for later calls */
        tyb_set_error("cudaPointerGetAttributes: %s", cudaGetErrorString(e));
        return -1;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

int tyb_residency(const void *p, void **view)
{
    struct cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        tyb_set_error("cudaPointerGetAttributes: %s", cudaGetErrorString(e));
        return -1;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        *view = (void *)p;
        return TYB_MEM_DEVICE;
    }
    if (attr.type == cudaMemoryTypeHost && attr.devicePointer) {
        /* devicePointer is the mapping of the allocation's base view; keep p's offset. */
        *view = (char *)attr.devicePointer + ((const char *)p - (const char *)attr.hostPointer);
        return TYB_MEM_PINNED;
    }
    *view = NULL;
    return TYB_MEM_HOST;
}

/* ---- device and page-locked allocations --------------------------------------------- */

/* Host-side failure injection for tests of the allocation-failure paths: with
 * TYB_FAULT_ALLOC=N in the environment (N > 0, optionally followed by non-digit text), the N-th
 * allocation through tyb_dev_alloc / tyb_host_alloc after the variable takes that value fails as
 * if the memory were exhausted.  A new value restarts the count; unset, nothing fails. */
static pthread_mutex_t g_fault_lock = PTHREAD_MUTEX_INITIALIZER;
static char g_fault_seen[64];
static long g_fault_count;

static int fault_now(void)
{
    const char *v = getenv("TYB_FAULT_ALLOC");
    int fail = 0;
    pthread_mutex_lock(&g_fault_lock);
    if (!v || !*v) {
        g_fault_seen[0] = '\0';
        g_fault_count = 0;
    } else {
        if (strncmp(v, g_fault_seen, sizeof g_fault_seen) != 0) {
            snprintf(g_fault_seen, sizeof g_fault_seen, "%s", v);
            g_fault_count = 0;
        }
        const long n = strtol(v, NULL, 10);
        fail = n > 0 && ++g_fault_count == n;
    }
    pthread_mutex_unlock(&g_fault_lock);
    return fail;
}

int tyb_dev_alloc(void **p, size_t bytes, const char *what)
{
    *p = NULL;
    if (fault_now()) {
        tyb_set_error("%s: %s (injected by TYB_FAULT_ALLOC)", what, cudaGetErrorString(cudaErrorMemoryAllocation));
        return 0;
    }
    if (!tyb_cuda_ok(cudaMalloc(p, bytes), what)) {
        *p = NULL;
        return 0;
    }
    return 1;
}

int tyb_host_alloc(void **p, size_t bytes, unsigned int flags, const char *what)
{
    *p = NULL;
    if (fault_now()) {
        tyb_set_error("%s: %s (injected by TYB_FAULT_ALLOC)", what, cudaGetErrorString(cudaErrorMemoryAllocation));
        return 0;
    }
    if (!tyb_cuda_ok(cudaHostAlloc(p, bytes, flags), what)) {
        *p = NULL;
        return 0;
    }
    return 1;
}

/* ---- workspace: per device ---------------------------------------------------------- */

#define TYB_MAX_DEVICES 64
static pthread_mutex_t g_ws_lock = PTHREAD_MUTEX_INITIALIZER;
static void *g_ws_ptr[TYB_MAX_DEVICES][TYB_WS_COUNT];
static size_t g_ws_size[TYB_MAX_DEVICES][TYB_WS_COUNT];

void *tyb_workspace(int slot, size_t bytes)
{
    int dev = 0;
    if (!tyb_cuda_ok(cudaGetDevice(&dev), "workspace")) return NULL;
    if (dev < 0 || dev >= TYB_MAX_DEVICES) {
        tyb_set_error("workspace: device %d beyond the %d this library tracks", dev, TYB_MAX_DEVICES);
        return NULL;
    }
    void *p = NULL;
    pthread_mutex_lock(&g_ws_lock);
    if (g_ws_size[dev][slot] >= bytes && g_ws_ptr[dev][slot]) {
        p = g_ws_ptr[dev][slot];
    } else {
        if (g_ws_ptr[dev][slot]) {
            cudaDeviceSynchronize(); /* the smaller buffer may still be in use on this device */
            cudaFree(g_ws_ptr[dev][slot]);
            g_ws_ptr[dev][slot] = NULL;
            g_ws_size[dev][slot] = 0;
        }
        size_t want = bytes < 4096 ? 4096 : bytes;
        if (tyb_dev_alloc(&p, want, "workspace cudaMalloc")) {
            /* Counters and tickets must start at zero. */
            if (!tyb_cuda_ok(cudaMemset(p, 0, want), "workspace cudaMemset")) {
                cudaFree(p);
                p = NULL;
            } else {
                g_ws_ptr[dev][slot] = p;
                g_ws_size[dev][slot] = want;
            }
        }
    }
    pthread_mutex_unlock(&g_ws_lock);
    return p;
}

int attn_workspace_reserve(int max_tokens, int max_batch, int max_kv_len)
{
    if (max_tokens < 0 || max_batch < 0 || max_kv_len < 0) {
        tyb_set_error("attn_workspace_reserve: negative size");
        return 1;
    }
    const size_t tok = (size_t)(max_tokens > max_batch ? max_tokens : max_batch);
    const size_t q_bytes = tok * TYB_Q_FLOATS * sizeof(float);
    const size_t kv_bytes = (size_t)max_tokens * TYB_ROW_FLOATS * sizeof(float);
    /* the prefill output staging doubles as the staging of host K and V rows */
    const size_t o_bytes = q_bytes > 2 * kv_bytes ? q_bytes : 2 * kv_bytes;
    size_t part = 0, desc = 0, cnt = 0;
    if (max_batch > 0 && max_kv_len > 0) {
        int chunk = 0, nsplit = 0, nsplit32 = 0;
        tyb_decode_plan(max_batch, max_kv_len, TYB_BF16, &chunk, &nsplit);
        tyb_decode_plan(max_batch, max_kv_len, TYB_F32, &chunk, &nsplit32);
        if (nsplit32 > nsplit) nsplit = nsplit32;
        part = tyb_decode_partial_floats(max_batch, nsplit) * sizeof(float);
        desc = tyb_decode_maps_bytes(max_batch) + sizeof(tyb_seq_kv) * (size_t)max_batch;
        cnt = sizeof(unsigned int) * (size_t)max_batch * KV_NUM_KV_HEADS;
    }
    const size_t want[TYB_WS_COUNT] = {[TYB_WS_Q] = q_bytes, [TYB_WS_K] = kv_bytes, [TYB_WS_V] = kv_bytes,
                                       [TYB_WS_OUT] = o_bytes, [TYB_WS_PARTIALS] = part, [TYB_WS_COUNTERS] = cnt,
                                       [TYB_WS_DESC] = desc};
    for (int s = 0; s < TYB_WS_COUNT; s++)
        if (want[s] && !tyb_workspace(s, want[s])) return 1;
    return 0;
}

int attn_set_wait_limit_ns(unsigned long long ns)
{
    if (ns < 1000ull) {
        tyb_set_error("attn_set_wait_limit_ns: limit %llu ns is below 1000", ns);
        return 1;
    }
    return tyb_cuda_ok(tyb_set_wait_limit(ns), "attn_set_wait_limit_ns") ? 0 : 1;
}

/* ---- registry of scratch device buffers ------------------------------------------- */

#define TYB_REG_MAX 256
static pthread_mutex_t g_reg_lock = PTHREAD_MUTEX_INITIALIZER;
static const void *g_reg_ptr[TYB_REG_MAX];
static size_t g_reg_size[TYB_REG_MAX];

void tyb_registry_add(const void *p, size_t bytes)
{
    pthread_mutex_lock(&g_reg_lock);
    for (int i = 0; i < TYB_REG_MAX; i++)
        if (!g_reg_ptr[i]) {
            g_reg_ptr[i] = p;
            g_reg_size[i] = bytes;
            break;
        }
    pthread_mutex_unlock(&g_reg_lock);
}

void tyb_registry_remove(const void *p)
{
    pthread_mutex_lock(&g_reg_lock);
    for (int i = 0; i < TYB_REG_MAX; i++)
        if (g_reg_ptr[i] == p) {
            g_reg_ptr[i] = NULL;
            g_reg_size[i] = 0;
        }
    pthread_mutex_unlock(&g_reg_lock);
}

size_t tyb_registry_size(const void *p)
{
    size_t n = 0;
    pthread_mutex_lock(&g_reg_lock);
    for (int i = 0; i < TYB_REG_MAX; i++)
        if (p && g_reg_ptr[i] == p) n = g_reg_size[i];
    pthread_mutex_unlock(&g_reg_lock);
    return n;
}

/* ---- rows written by the previous launch ------------------------------------------ */

static _Thread_local struct {
    const void *cache;
    int layer;
    int lo;
    void *stream;
    int valid;
} g_last_write;

void tyb_note_write(const void *cache, int layer, int lo, void *stream)
{
    g_last_write.cache = cache;
    g_last_write.layer = layer;
    g_last_write.lo = lo;
    g_last_write.stream = stream;
    g_last_write.valid = 1;
}

void tyb_note_nowrite(void *stream)
{
    if (g_last_write.stream == stream) g_last_write.valid = 0;
}

int tyb_prefetch_rows(const void *cache, int layer, int rows)
{
    if (g_last_write.valid && g_last_write.cache == cache && g_last_write.layer == layer)
        return g_last_write.lo < rows ? g_last_write.lo : rows;
    return rows;
}

/* ---- synchronisation + status ----------------------------------------------------- */

int tyb_finish(void *stream, const char *what)
{
    unsigned int bits = 0;
    volatile unsigned int *mirror = tyb_status_mirror_host();
    if (mirror) {
        /* Kernels flag the mirror whenever they raise a status bit: an unflagged mirror after
         * the synchronisation means the status word is clear, with no read-back. */
        if (!tyb_cuda_ok(cudaStreamSynchronize((cudaStream_t)stream), what)) return 0;
        if (*mirror == 0u) {
            if (g_last_write.stream == stream) g_last_write.valid = 0;
            return 1;
        }
        *mirror = 0u;
    }
    int e = tyb_status_fetch(&bits, stream);
    if (!tyb_cuda_ok(e, what)) return 0;
    if (g_last_write.stream == stream) g_last_write.valid = 0; /* everything queued is done */
    if (bits) {
        tyb_set_error("%s: device status 0x%x (%s%s)", what, bits,
                      (bits & TYB_STATUS_WAIT_TIMEOUT) ? "wait timed out " : "",
                      (bits & TYB_STATUS_BAD_ARGUMENT) ? "index check failed" : "");
        return 0;
    }
    return 1;
}

int attn_sync(void) { return tyb_finish(g_stream, "attn_sync") ? 0 : 1; }

/* A blocking decode call with a host output returns once the output is there, not once the
 * launch has retired: measured on a B200 (4K-row BF16 decode, page-locked buffers), a host
 * waiting in cudaStreamSynchronize saw the launch complete ~3 us after a host polling the output
 * saw the last word land.  The output is filled with TYB_UNWRITTEN before the launch -- a NaN
 * whose sign bit is set, which GPU arithmetic never produces (it returns the canonical NaN
 * 0x7FFFFFFF) -- and each word is written once by the kernel with a 16-byte store, so the call
 * waits until no word holds the pattern.  No fence or flag is needed in the kernel: the words
 * themselves are the signal.  Every 1024 rounds the stream is queried: if it went idle (or
 * failed) first, or a kernel raised a status bit, the full synchronisation reports the outcome. */
void tyb_mark_unwritten(float *out, size_t n)
{
    unsigned int *w = (unsigned int *)out;
    for (size_t i = 0; i < n; i++) w[i] = TYB_UNWRITTEN;
}

int tyb_wait_output(const float *out, size_t n, void *stream, const char *what)
{
    const unsigned int *w = (const unsigned int *)out;
    volatile unsigned int *mirror = tyb_status_mirror_host();
    size_t i = 0; /* words [0, i) are written */
    for (unsigned long spin = 1;; spin++) {
        while (i < n && __atomic_load_n(&w[i], __ATOMIC_ACQUIRE) != TYB_UNWRITTEN) i++;
        if (mirror && *mirror) break;
        if (i == n) return 1;
        if ((spin & 1023u) == 0u && cudaStreamQuery((cudaStream_t)stream) != cudaErrorNotReady) break;
    }
    return tyb_finish(stream, what);
}
