/*
 * storage.c - the .magnetron tensor file format (storage v1) with device-resident data.
 *
 * Format (magnetron/magnetron.c:2688-3011), all integers little-endian:
 *   file header   20 B: u64 magic "magtron!", u32 version, u32 tensor count, u32 user data (0)
 *   tensor header 116 B each, all headers first: 64 B name, u32 aux = flags<<16 | dtype<<8 | rank,
 *                 6 x u64 shape
 *   data          each tensor's f32 elements in header order, no padding
 * The reference serialises to and from host memory only (it asserts a CPU context at
 * magnetron/magnetron.c:2878 and :2912).  Here the headers are built and checked on the
 * host, and tensor data moves between the file and HBM in 8 MiB chunks through pinned
 * buffers, two per lane, so a lane's pread/pwrite of one chunk overlaps the DMA of the
 * other and the file is never staged whole in host memory.  Loads run 12 lanes (page-cache
 * reads of one file proceed in parallel); saves run one, because buffered writes to one
 * file serialise on the inode in common filesystems, and overwrite the old file in place
 * (trimmed at the end) instead of truncating it first, which skips freeing and
 * reallocating its blocks.
 *
 * The parser applies the reference reader's checks in its order and rejects what it
 * rejects (mag_sto_read_buffered returns NULL there); where the reference aborts on a
 * data region that runs past the end of the buffer (mag_assert2 at :2914) this returns
 * MAG_CUDA_E_INVALID.
 */
#include "mag_cuda_abi.h"
#include "magnetron_cuda.h"
#include "mcu_device.h"

#include <cuda_runtime_api.h>
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#define STO_FILE_HDR 20u
#define STO_TENSOR_HDR 116u
#define STO_VERSION 1u     /* MAG_STORAGE_VERSION (magnetron/magnetron.h:51) */
#define STO_LIB_VERSION 1u /* MAG_VERSION = mag_version_pack(0, 1) (magnetron/magnetron.h:47-50), the reader's bound */
#define STO_FLAG_BITS 4    /* MAG_TFLAG_LEN (magnetron/magnetron_internal.h:423) */
#define STO_DTYPES 1       /* MAG_DTYPE_COUNT_: f32 only (magnetron/magnetron.h:123-126) */

#define STO_CHUNK ((size_t)8 << 20)
#define STO_THREADS 12 /* lanes for loads: page-cache reads run in parallel */
#define STO_MAX_DEVICES 64

/* ------------------------------------------------------- byte order --- */

static void put_u32(uint8_t* p, uint32_t x) {
    for (int i = 0; i < 4; ++i) p[i] = (uint8_t)(x >> (8 * i));
}
static void put_u64(uint8_t* p, uint64_t x) {
    for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(x >> (8 * i));
}
static uint32_t get_u32(const uint8_t* p) {
    uint32_t x = 0;
    for (int i = 0; i < 4; ++i) x |= (uint32_t)p[i] << (8 * i);
    return x;
}
static uint64_t get_u64(const uint8_t* p) {
    uint64_t x = 0;
    for (int i = 0; i < 8; ++i) x |= (uint64_t)p[i] << (8 * i);
    return x;
}

/* ------------------------------------------------------------ parser --- */

/* mag_sto_read_buffered's header phase (magnetron/magnetron.c:2891-2911) over the first
 * `avail` bytes of a file of `total` bytes; data offsets follow the headers in order. */
int mag_cuda_sto_parse(const void* buf, size_t avail, size_t total, mag_cuda_sto_entry* entries, uint32_t cap,
                       uint32_t* n_tensors, uint32_t* version) {
    const uint8_t* b = (const uint8_t*)buf;
    if (!b || !n_tensors || !version || avail > total) return MAG_CUDA_E_INVALID;
    if (total <= STO_FILE_HDR + STO_TENSOR_HDR + 1) return MAG_CUDA_E_INVALID; /* :2892 */
    if (avail < STO_FILE_HDR) return MAG_CUDA_E_INVALID;
    if (memcmp(b, "magtron!", 8) != 0) return MAG_CUDA_E_INVALID; /* :2755 */
    const uint32_t ver = get_u32(b + 8), n = get_u32(b + 12);
    if (!ver || ver > STO_LIB_VERSION) return MAG_CUDA_E_INVALID; /* :2898 */
    if (!n) return MAG_CUDA_E_INVALID;                            /* :2899 */
    if (ver != STO_VERSION) return MAG_CUDA_E_INVALID;            /* only v1 headers exist (:2806) */
    uint64_t pos = STO_FILE_HDR;
    for (uint32_t i = 0; i < n; ++i, pos += STO_TENSOR_HDR) {
        if (!(pos + STO_TENSOR_HDR < total)) return MAG_CUDA_E_INVALID; /* :2804, strict */
        if (pos + STO_TENSOR_HDR > avail) return MAG_CUDA_E_INVALID;
        const uint8_t* h = b + pos;
        const uint32_t aux = get_u32(h + 64);
        const uint32_t flags = (aux >> 16) & 0xff, dtype = (aux >> 8) & 0xff, rank = aux & 0xff;
        if (flags & ~((1u << STO_FLAG_BITS) - 1)) return MAG_CUDA_E_INVALID; /* :2815-2817 */
        if (dtype >= STO_DTYPES) return MAG_CUDA_E_INVALID;
        if (rank < 1 || rank > 6) return MAG_CUDA_E_INVALID;
        int64_t sh[6];
        for (int k = 0; k < 6; ++k) {
            const uint64_t u = get_u64(h + 68 + 8 * k);
            if (u < 1 || u > (uint64_t)INT64_MAX) return MAG_CUDA_E_INVALID; /* :2820 */
            sh[k] = (int64_t)u;
        }
        int64_t prod = sh[0]; /* :2823-2827, strict */
        for (int k = 1; k < 6; ++k) {
            if (!(INT64_MAX / sh[k] > prod)) return MAG_CUDA_E_INVALID;
            prod *= sh[k];
        }
        if (entries && i < cap) {
            mag_cuda_sto_entry* e = &entries[i];
            memcpy(e->name, h, 64);
            e->name[63] = '\0';
            e->flags = flags;
            e->dtype = dtype;
            e->rank = rank;
            memcpy(e->shape, sh, sizeof(sh));
        }
    }
    /* data phase (:2912-2916): each region must lie inside the file */
    for (uint32_t i = 0; i < n; ++i) {
        const uint8_t* h = b + STO_FILE_HDR + (uint64_t)i * STO_TENSOR_HDR;
        uint64_t bytes = 4; /* f32; the overflow checks above bound the element count by INT64_MAX */
        for (int k = 0; k < 6; ++k) {
            const uint64_t d = get_u64(h + 68 + 8 * k);
            if (bytes > UINT64_MAX / d) return MAG_CUDA_E_INVALID;
            bytes *= d;
        }
        if (bytes > total || pos > total - bytes) return MAG_CUDA_E_INVALID;
        if (entries && i < cap) {
            entries[i].offset = pos;
            entries[i].bytes = bytes;
        }
        pos += bytes;
    }
    *n_tensors = n;
    *version = ver;
    return 0;
}

/* mag_sto_write_file_header + mag_sto_write_tensor_header (magnetron/magnetron.c:2729-2785). */
static int sto_header(const mag_tensor_t* const* ts, uint32_t n, uint8_t** out, size_t* hdr, uint64_t* total) {
    const size_t h = STO_FILE_HDR + (size_t)n * STO_TENSOR_HDR;
    uint8_t* p = (uint8_t*)calloc(1, h);
    if (!p) return MAG_CUDA_E_INVALID;
    memcpy(p, "magtron!", 8);
    put_u32(p + 8, STO_VERSION);
    put_u32(p + 12, n);
    put_u32(p + 16, 0);
    uint64_t tot = h;
    for (uint32_t i = 0; i < n; ++i) {
        const mag_tensor_t* t = ts[i];
        uint8_t* q = p + STO_FILE_HDR + (size_t)i * STO_TENSOR_HDR;
        if (!t || t->dtype != 0 || t->rank < 1 || t->rank > 6) goto bad;
        memcpy(q, t->name, 64);
        put_u32(q + 64, ((uint32_t)(t->flags & 0xff) << 16) | ((uint32_t)(t->dtype & 0xff) << 8) |
                            (uint32_t)(t->rank & 0xff));
        for (int k = 0; k < 6; ++k) {
            if (t->shape[k] < 1) goto bad; /* :2779 */
            put_u64(q + 68 + 8 * k, (uint64_t)t->shape[k]);
        }
        const uint64_t bytes = (uint64_t)t->numel * 4;
        if (!t->numel || bytes > t->storage.size) goto bad; /* :2842 size > 0 */
        tot += bytes;
    }
    *out = p;
    *hdr = h;
    *total = tot;
    return 0;
bad:
    free(p);
    return MAG_CUDA_E_INVALID;
}

int mag_cuda_sto_write_header(const mag_tensor_t* const* tensors, uint32_t n, void* buf, size_t cap, size_t* size) {
    if (!tensors || !n || !size) return MAG_CUDA_E_INVALID;
    uint8_t* p;
    size_t h;
    uint64_t tot;
    int rc = sto_header(tensors, n, &p, &h, &tot);
    if (rc) return rc;
    *size = h;
    if (buf && cap >= h) memcpy(buf, p, h);
    free(p);
    return buf && cap < h ? MAG_CUDA_E_INVALID : 0;
}

/* mag_sto_has_mag_ext (magnetron/magnetron.c:2925-2929). */
static int has_ext(const char* path) {
    if (!path || strlen(path) < sizeof(".magnetron")) return 0;
    const char* dot = strrchr(path, '.');
    return dot && !strcmp(dot, ".magnetron");
}

/* ------------------------------------------------------- I/O engine --- */

typedef struct sto_lane {
    void* buf[2];
    cudaEvent_t ev[2];
    cudaStream_t st;
} sto_lane;

typedef struct sto_pool {
    pthread_mutex_t mu;
    int ready;
    sto_lane lane[STO_THREADS];
} sto_pool;

static sto_pool g_pools[STO_MAX_DEVICES];
static pthread_once_t g_pools_once = PTHREAD_ONCE_INIT;
static void pools_init(void) {
    for (int i = 0; i < STO_MAX_DEVICES; ++i) pthread_mutex_init(&g_pools[i].mu, NULL);
}

/* Pinned buffers, events and streams of one device, created on first use and kept. */
static int pool_get(int ordinal, sto_pool** out) {
    if (ordinal < 0 || ordinal >= STO_MAX_DEVICES) return MAG_CUDA_E_INVALID;
    pthread_once(&g_pools_once, pools_init);
    sto_pool* p = &g_pools[ordinal];
    pthread_mutex_lock(&p->mu);
    int rc = 0;
    if (!p->ready) {
        for (int t = 0; t < STO_THREADS && !rc; ++t) {
            sto_lane* l = &p->lane[t];
            if (cudaStreamCreateWithFlags(&l->st, cudaStreamNonBlocking) != cudaSuccess) rc = MAG_CUDA_E_IO;
            for (int s = 0; s < 2 && !rc; ++s) {
                if (cudaHostAlloc(&l->buf[s], STO_CHUNK, cudaHostAllocDefault) != cudaSuccess ||
                    cudaEventCreateWithFlags(&l->ev[s], cudaEventDisableTiming) != cudaSuccess)
                    rc = MAG_CUDA_E_IO;
            }
        }
        if (!rc) p->ready = 1;
    }
    pthread_mutex_unlock(&p->mu);
    *out = p;
    return rc;
}

typedef struct sto_chunk {
    char* dev;
    uint64_t off;
    size_t len;
} sto_chunk;

typedef struct sto_job {
    int fd;
    int save;
    int ordinal;
    sto_pool* pool;
    const sto_chunk* chunks;
    size_t n_chunks;
    int n_threads;
    atomic_int err;
} sto_job;

typedef struct sto_arg {
    sto_job* job;
    int lane;
} sto_arg;

static int full_pread(int fd, void* buf, size_t len, uint64_t off) {
    char* p = (char*)buf;
    while (len) {
        ssize_t r = pread(fd, p, len, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return -1;
        p += r;
        off += (uint64_t)r;
        len -= (size_t)r;
    }
    return 0;
}

static int full_pwrite(int fd, const void* buf, size_t len, uint64_t off) {
    const char* p = (const char*)buf;
    while (len) {
        ssize_t r = pwrite(fd, p, len, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return -1;
        p += r;
        off += (uint64_t)r;
        len -= (size_t)r;
    }
    return 0;
}

/* One lane: chunks lane, lane + T, ...; two pinned buffers alternate, so the file
 * transfer of one chunk runs while the other's DMA is in flight. */
static void* sto_lane_run(void* argp) {
    sto_arg* a = (sto_arg*)argp;
    sto_job* j = a->job;
    sto_lane* l = &j->pool->lane[a->lane];
    if (cudaSetDevice(j->ordinal) != cudaSuccess) {
        atomic_store(&j->err, MAG_CUDA_E_IO);
        return NULL;
    }
    const size_t T = (size_t)j->n_threads;
    int rc = 0;
    if (!j->save) {
        int k = 0;
        for (size_t c = (size_t)a->lane; c < j->n_chunks && !rc && !atomic_load(&j->err); c += T, k ^= 1) {
            const sto_chunk* ch = &j->chunks[c];
            if (cudaEventSynchronize(l->ev[k]) != cudaSuccess) rc = MAG_CUDA_E_IO;
            else if (full_pread(j->fd, l->buf[k], ch->len, ch->off)) rc = MAG_CUDA_E_IO;
            else if (cudaMemcpyAsync(ch->dev, l->buf[k], ch->len, cudaMemcpyHostToDevice, l->st) != cudaSuccess ||
                     cudaEventRecord(l->ev[k], l->st) != cudaSuccess)
                rc = MAG_CUDA_E_IO;
        }
    } else {
        size_t c = (size_t)a->lane;
        int k = 0;
        if (c < j->n_chunks) {
            const sto_chunk* ch = &j->chunks[c];
            if (cudaMemcpyAsync(l->buf[0], ch->dev, ch->len, cudaMemcpyDeviceToHost, l->st) != cudaSuccess ||
                cudaEventRecord(l->ev[0], l->st) != cudaSuccess)
                rc = MAG_CUDA_E_IO;
        }
        for (; c < j->n_chunks && !rc && !atomic_load(&j->err); c += T, k ^= 1) {
            const size_t nx = c + T;
            if (nx < j->n_chunks) { /* the other buffer's last write has returned */
                const sto_chunk* cn = &j->chunks[nx];
                if (cudaMemcpyAsync(l->buf[k ^ 1], cn->dev, cn->len, cudaMemcpyDeviceToHost, l->st) != cudaSuccess ||
                    cudaEventRecord(l->ev[k ^ 1], l->st) != cudaSuccess) {
                    rc = MAG_CUDA_E_IO;
                    break;
                }
            }
            const sto_chunk* ch = &j->chunks[c];
            if (cudaEventSynchronize(l->ev[k]) != cudaSuccess || full_pwrite(j->fd, l->buf[k], ch->len, ch->off))
                rc = MAG_CUDA_E_IO;
        }
    }
    if (cudaStreamSynchronize(l->st) != cudaSuccess && !rc) rc = MAG_CUDA_E_IO;
    if (rc) atomic_store(&j->err, rc);
    return NULL;
}

/* Moves every chunk between the file and device memory with up to STO_THREADS lanes. */
static int sto_stream(int ordinal, int fd, int save, const sto_chunk* chunks, size_t n_chunks) {
    if (!n_chunks) return 0;
    sto_pool* pool;
    int rc = pool_get(ordinal, &pool);
    if (rc) return rc;
    sto_job j = {fd, save, ordinal, pool, chunks, n_chunks, 0, 0};
    const size_t lanes = save ? 1 : STO_THREADS;
    j.n_threads = (int)(n_chunks < lanes ? n_chunks : lanes);
    atomic_init(&j.err, 0);
    pthread_t th[STO_THREADS];
    sto_arg args[STO_THREADS];
    int started = 0;
    for (int t = 0; t < j.n_threads; ++t) {
        args[t] = (sto_arg){&j, t};
        if (t == 0) continue;
        if (pthread_create(&th[t], NULL, sto_lane_run, &args[t])) {
            atomic_store(&j.err, MAG_CUDA_E_IO);
            break;
        }
        started = t;
    }
    int prev = ordinal;
    cudaGetDevice(&prev);
    sto_lane_run(&args[0]); /* the calling thread is lane 0 */
    for (int t = 1; t <= started; ++t) pthread_join(th[t], NULL);
    cudaSetDevice(prev);
    return atomic_load(&j.err);
}

/* Chunk list for regions laid out back to back from file offset `off`. */
static int make_chunks(char* const* devs, const uint64_t* bytes, uint32_t n, uint64_t off, sto_chunk** out,
                       size_t* n_out) {
    size_t cnt = 0;
    for (uint32_t i = 0; i < n; ++i) cnt += (size_t)((bytes[i] + STO_CHUNK - 1) / STO_CHUNK);
    sto_chunk* c = (sto_chunk*)malloc((cnt ? cnt : 1) * sizeof(sto_chunk));
    if (!c) return MAG_CUDA_E_INVALID;
    size_t k = 0;
    for (uint32_t i = 0; i < n; ++i) {
        for (uint64_t o = 0; o < bytes[i]; o += STO_CHUNK) {
            const uint64_t len = bytes[i] - o < STO_CHUNK ? bytes[i] - o : STO_CHUNK;
            c[k++] = (sto_chunk){devs[i] + o, off + o, (size_t)len};
        }
        off += bytes[i];
    }
    *out = c;
    *n_out = cnt;
    return 0;
}

/* ------------------------------------------------------------- public --- */

int mag_cuda_tensor_save(mag_compute_device_t* dvc, const char* path, const mag_tensor_t* const* tensors, uint32_t n) {
    if (!dvc || !tensors || !n || !has_ext(path)) return MAG_CUDA_E_INVALID;
    uint8_t* hdr;
    size_t h;
    uint64_t total;
    int rc = sto_header(tensors, n, &hdr, &h, &total);
    if (rc) return rc;
    char** devs = (char**)malloc(n * sizeof(char*));
    uint64_t* bytes = (uint64_t*)malloc(n * sizeof(uint64_t));
    sto_chunk* chunks = NULL;
    size_t n_chunks = 0;
    int fd = -1;
    if (!devs || !bytes) {
        rc = MAG_CUDA_E_INVALID;
        goto done;
    }
    for (uint32_t i = 0; i < n; ++i) {
        devs[i] = (char*)tensors[i]->storage.base;
        bytes[i] = (uint64_t)tensors[i]->numel * 4;
        mcu_dev_in(dvc, devs[i]); /* a never-written buffer is cleared first: it reads as zero */
    }
    rc = mcu_dev_sync(dvc); /* results of queued ops are complete before the copies start */
    if (rc) goto done;
    if ((rc = make_chunks(devs, bytes, n, h, &chunks, &n_chunks))) goto done;
    fd = open(path, O_WRONLY | O_CREAT, 0644);
    if (fd < 0 || full_pwrite(fd, hdr, h, 0)) {
        rc = MAG_CUDA_E_IO;
        goto done;
    }
    rc = sto_stream(mcu_dev_ordinal(dvc), fd, 1, chunks, n_chunks);
    if (!rc && ftruncate(fd, (off_t)total)) rc = MAG_CUDA_E_IO; /* drop what an older, longer file left */
done:
    if (fd >= 0 && close(fd) && !rc) rc = MAG_CUDA_E_IO;
    free(chunks);
    free(devs);
    free(bytes);
    free(hdr);
    return rc;
}

static int read_directory_fd(int fd, uint64_t total, mag_cuda_sto_entry* entries, uint32_t cap, uint32_t* n,
                             uint32_t* version) {
    uint8_t fh[STO_FILE_HDR];
    if (total < STO_FILE_HDR || full_pread(fd, fh, STO_FILE_HDR, 0)) return MAG_CUDA_E_INVALID;
    const uint64_t cnt = get_u32(fh + 12);
    if (cnt > (total - STO_FILE_HDR) / STO_TENSOR_HDR) return MAG_CUDA_E_INVALID; /* headers cannot fit */
    const uint64_t avail = STO_FILE_HDR + cnt * STO_TENSOR_HDR;
    uint8_t* buf = (uint8_t*)malloc((size_t)avail);
    if (!buf) return MAG_CUDA_E_INVALID;
    int rc = full_pread(fd, buf, (size_t)avail, 0) ? MAG_CUDA_E_IO : 0;
    if (!rc) {
        /* all headers are needed for the offsets: parse into a full table, copy out cap */
        mag_cuda_sto_entry* all = (mag_cuda_sto_entry*)calloc(cnt ? cnt : 1, sizeof(mag_cuda_sto_entry));
        if (!all) rc = MAG_CUDA_E_INVALID;
        else {
            rc = mag_cuda_sto_parse(buf, (size_t)avail, (size_t)total, all, (uint32_t)cnt, n, version);
            if (!rc && entries) memcpy(entries, all, (size_t)(cap < *n ? cap : *n) * sizeof(*all));
            free(all);
        }
    }
    free(buf);
    return rc;
}

int mag_cuda_sto_read_directory(const char* path, mag_cuda_sto_entry* entries, uint32_t cap, uint32_t* n_tensors,
                                uint32_t* version) {
    if (!has_ext(path) || !n_tensors || !version) return MAG_CUDA_E_INVALID;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return MAG_CUDA_E_IO;
    struct stat sb;
    int rc = fstat(fd, &sb) ? MAG_CUDA_E_IO
                            : read_directory_fd(fd, (uint64_t)sb.st_size, entries, cap, n_tensors, version);
    close(fd);
    return rc;
}

int mag_cuda_tensor_load(mag_compute_device_t* dvc, const char* path, mag_tensor_t* const* tensors, uint32_t n) {
    if (!dvc || !tensors || !has_ext(path)) return MAG_CUDA_E_INVALID;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return MAG_CUDA_E_IO;
    struct stat sb;
    uint32_t cnt = 0, ver = 0;
    mag_cuda_sto_entry* e = NULL;
    char** devs = NULL;
    uint64_t* bytes = NULL;
    sto_chunk* chunks = NULL;
    size_t n_chunks = 0;
    int rc = fstat(fd, &sb) ? MAG_CUDA_E_IO : 0;
    if (!rc) {
        uint8_t fh[STO_FILE_HDR];
        rc = (uint64_t)sb.st_size >= STO_FILE_HDR && !full_pread(fd, fh, STO_FILE_HDR, 0) ? 0 : MAG_CUDA_E_INVALID;
        if (!rc) {
            cnt = get_u32(fh + 12);
            if (cnt > ((uint64_t)sb.st_size - STO_FILE_HDR) / STO_TENSOR_HDR) cnt = 0; /* rejected below */
            e = (mag_cuda_sto_entry*)calloc(cnt ? cnt : 1, sizeof(*e));
            rc = e ? read_directory_fd(fd, (uint64_t)sb.st_size, e, cnt, &cnt, &ver) : MAG_CUDA_E_INVALID;
        }
    }
    if (!rc && (n == 0 || n > cnt)) rc = MAG_CUDA_E_INVALID;
    if (!rc) {
        devs = (char**)malloc(n * sizeof(char*));
        bytes = (uint64_t*)malloc(n * sizeof(uint64_t));
        if (!devs || !bytes) rc = MAG_CUDA_E_INVALID;
    }
    for (uint32_t i = 0; !rc && i < n; ++i) { /* destination shapes must be the stored ones */
        const mag_tensor_t* t = tensors[i];
        if (!t || t->dtype != (int32_t)e[i].dtype || t->rank != e[i].rank || memcmp(t->shape, e[i].shape, 48) ||
            (uint64_t)t->numel * 4 != e[i].bytes || e[i].bytes > t->storage.size)
            rc = MAG_CUDA_E_INVALID;
        else {
            devs[i] = (char*)t->storage.base;
            bytes[i] = e[i].bytes;
        }
    }
    if (!rc) { /* regions are consecutive: one chunk list per tensor at its own offset */
        for (uint32_t i = 0; !rc && i < n; ++i) {
            sto_chunk* c;
            size_t m;
            if ((rc = make_chunks(&devs[i], &bytes[i], 1, e[i].offset, &c, &m))) break;
            sto_chunk* grown = (sto_chunk*)realloc(chunks, (n_chunks + m + 1) * sizeof(sto_chunk));
            if (!grown) {
                free(c);
                rc = MAG_CUDA_E_INVALID;
                break;
            }
            chunks = grown;
            memcpy(chunks + n_chunks, c, m * sizeof(sto_chunk));
            n_chunks += m;
            free(c);
        }
    }
    if (!rc) {
        for (uint32_t i = 0; i < n; ++i) mcu_dev_out(dvc, devs[i], (size_t)bytes[i]);
        rc = mcu_dev_sync(dvc); /* earlier ops that read the destinations finish before they are overwritten */
        if (!rc) rc = sto_stream(mcu_dev_ordinal(dvc), fd, 0, chunks, n_chunks);
    }
    if (!rc) { /* the reader names the tensor and sets its flags (magnetron/magnetron.c:2907-2908) */
        for (uint32_t i = 0; i < n; ++i) {
            snprintf(tensors[i]->name, sizeof(tensors[i]->name), "%s", e[i].name);
            tensors[i]->flags = (int32_t)e[i].flags;
        }
    }
    close(fd);
    free(chunks);
    free(devs);
    free(bytes);
    free(e);
    return rc;
}
