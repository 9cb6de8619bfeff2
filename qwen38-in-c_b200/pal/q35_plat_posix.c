/* POSIX / Linux implementation of the engine's platform layer
 * (include/q35_plat.h, the interface of qwen35-c/src/q35_plat.h).
 *
 * What each entry point does here, where the reference's Windows layer
 * (qwen35-c/src/q35_plat_win.c) used a Win32 call:
 *   read_file        open + fstat + read loop, NUL-terminated copy
 *   aligned_alloc    posix_memalign
 *   large_alloc      a 2 MB huge-page mapping (MAP_HUGETLB) when the host has
 *                    reserved huge pages, else an anonymous mapping marked
 *                    MADV_HUGEPAGE (transparent huge pages) for sizes of at
 *                    least one huge page; NULL for smaller requests, as the
 *                    reference returns NULL when large pages are unavailable
 *   dir_*            opendir/readdir, regular files only
 *   mmap_ro          open + mmap(PROT_READ, MAP_PRIVATE), MADV_SEQUENTIAL
 *   mmap_prefetch    MADV_WILLNEED over the mapping, then one touch per page;
 *                    when libq35cuda is loaded in the process and the mapping
 *                    is a safetensors shard, its matmul weights are then
 *                    uploaded to the GPU (q35cu_preload_safetensors), so the
 *                    first forward pass does not upload on first touch
 *                    (Q35_PRELOAD=0 turns this off)
 *   avail_phys       MemAvailable of /proc/meminfo (sysconf fallback)
 *   peak_rss         getrusage ru_maxrss
 *   num_phys_cores   distinct (package, core) pairs of the CPUs this process
 *                    may run on (sysfs topology), online CPUs as fallback
 *   sockets          loopback TCP; send never raises SIGPIPE
 */
#define _GNU_SOURCE
#define _FILE_OFFSET_BITS 64

#include "q35_plat.h"

#include <arpa/inet.h>
#include <dirent.h>
#include <dlfcn.h>
#include <errno.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <pthread.h>
#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/resource.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#define Q35_API __attribute__((visibility("default")))

static const size_t kHuge = (size_t)2 << 20;

Q35_API void *q35_plat_read_file(const char *path, size_t *out_len)
{
    if (!path) return NULL;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return NULL;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || !S_ISREG(sb.st_mode) || sb.st_size < 0) {
        close(fd);
        return NULL;
    }
    const size_t n = (size_t)sb.st_size;
    char *buf = (char *)malloc(n + 1);
    if (!buf) {
        close(fd);
        return NULL;
    }
    size_t got = 0;
    while (got < n) {
        const ssize_t r = read(fd, buf + got, n - got);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) {
            free(buf);
            close(fd);
            return NULL;
        }
        got += (size_t)r;
    }
    close(fd);
    buf[n] = '\0';
    if (out_len) *out_len = n;
    return buf;
}

Q35_API void *q35_plat_aligned_alloc(size_t alignment, size_t size)
{
    void *p = NULL;
    if (alignment < sizeof(void *)) alignment = sizeof(void *);
    if (posix_memalign(&p, alignment, size ? size : 1) != 0) return NULL;
    return p;
}

Q35_API void q35_plat_aligned_free(void *p) { free(p); }
Q35_API void q35_plat_free(void *p) { free(p); }

/* large mappings handed out, so that large_free knows their lengths */
#define Q35_MAX_LARGE 256
static struct {
    void *p;
    size_t len;
} g_large[Q35_MAX_LARGE];
static pthread_mutex_t g_large_mu = PTHREAD_MUTEX_INITIALIZER;

Q35_API void *q35_plat_large_alloc(size_t size)
{
    if (size < kHuge) return NULL;
    const size_t len = (size + kHuge - 1) / kHuge * kHuge;
    void *p = mmap(NULL, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_HUGETLB, -1, 0);
    if (p == MAP_FAILED) {
        p = mmap(NULL, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
        if (p == MAP_FAILED) return NULL;
        if (madvise(p, len, MADV_HUGEPAGE) != 0) {  /* no transparent huge pages: not a large-page mapping */
            munmap(p, len);
            return NULL;
        }
    }
    pthread_mutex_lock(&g_large_mu);
    for (int i = 0; i < Q35_MAX_LARGE; ++i)
        if (!g_large[i].p) {
            g_large[i].p = p;
            g_large[i].len = len;
            pthread_mutex_unlock(&g_large_mu);
            return p;
        }
    pthread_mutex_unlock(&g_large_mu);
    munmap(p, len);  /* registry full: let the caller use its own allocator */
    return NULL;
}

Q35_API void q35_plat_large_free(void *p)
{
    if (!p) return;
    pthread_mutex_lock(&g_large_mu);
    for (int i = 0; i < Q35_MAX_LARGE; ++i)
        if (g_large[i].p == p) {
            munmap(p, g_large[i].len);
            g_large[i].p = NULL;
            g_large[i].len = 0;
            break;
        }
    pthread_mutex_unlock(&g_large_mu);
}

Q35_API double q35_plat_now(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

struct Q35PlatDir {
    DIR *dp;
    int fd;  /* dirfd, for fstatat when d_type is unknown */
};

Q35_API Q35PlatDir *q35_plat_dir_open(const char *dir)
{
    if (!dir) return NULL;
    DIR *dp = opendir(dir);
    if (!dp) return NULL;
    Q35PlatDir *d = (Q35PlatDir *)calloc(1, sizeof(*d));
    if (!d) {
        closedir(dp);
        return NULL;
    }
    d->dp = dp;
    d->fd = dirfd(dp);
    return d;
}

Q35_API const char *q35_plat_dir_next(Q35PlatDir *d)
{
    if (!d) return NULL;
    for (;;) {
        struct dirent *e = readdir(d->dp);
        if (!e) return NULL;
        if (e->d_type == DT_REG) return e->d_name;
        if (e->d_type == DT_UNKNOWN || e->d_type == DT_LNK) {  /* ask the file system */
            struct stat sb;
            if (fstatat(d->fd, e->d_name, &sb, 0) == 0 && S_ISREG(sb.st_mode)) return e->d_name;
        }
    }
}

Q35_API void q35_plat_dir_close(Q35PlatDir *d)
{
    if (!d) return;
    closedir(d->dp);
    free(d);
}

Q35_API int q35_plat_fseek64(FILE *f, int64_t offset, int whence) { return fseeko(f, (off_t)offset, whence); }
Q35_API int64_t q35_plat_ftell64(FILE *f) { return (int64_t)ftello(f); }

struct Q35PlatMmap {
    void *base;
    size_t len;
    int fd;
};

Q35_API Q35PlatMmap *q35_plat_mmap_ro(const char *path, const uint8_t **out_base)
{
    if (!path) return NULL;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return NULL;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || !S_ISREG(sb.st_mode) || sb.st_size <= 0) {
        close(fd);
        return NULL;
    }
    const size_t len = (size_t)sb.st_size;
    void *p = mmap(NULL, len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
        close(fd);
        return NULL;
    }
    madvise(p, len, MADV_SEQUENTIAL);
    Q35PlatMmap *m = (Q35PlatMmap *)calloc(1, sizeof(*m));
    if (!m) {
        munmap(p, len);
        close(fd);
        return NULL;
    }
    m->base = p;
    m->len = len;
    m->fd = fd;
    if (out_base) *out_base = (const uint8_t *)p;
    return m;
}

/* libq35cuda's preload entry points, when that library is in the process:
 * linked into the program, or opened with local symbol scope (a host
 * language's FFI) -- found by its soname without loading it */
typedef int (*preload_fn)(const void *, size_t);
typedef void (*forget_fn)(const void *, size_t);

static void *q35cuda_sym(const char *name)
{
    void *s = dlsym(RTLD_DEFAULT, name);
    if (s) return s;
    void *h = dlopen("libq35cuda.so", RTLD_NOLOAD | RTLD_LAZY);
    if (!h) return NULL;
    s = dlsym(h, name);
    dlclose(h);  /* drops only the reference RTLD_NOLOAD took */
    return s;
}

static int preload_enabled(void)
{
    const char *e = getenv("Q35_PRELOAD");
    return !(e && strcmp(e, "0") == 0);
}

Q35_API void q35_plat_munmap(Q35PlatMmap *m)
{
    if (!m) return;
    forget_fn forget = (forget_fn)q35cuda_sym("q35cu_preload_forget");
    if (forget && m->base) forget(m->base, m->len);
    if (m->base) munmap(m->base, m->len);
    if (m->fd >= 0) close(m->fd);
    free(m);
}

Q35_API void q35_plat_prefetch(const void *base, size_t len)
{
    if (!base || !len) return;
    const long pg = sysconf(_SC_PAGESIZE) > 0 ? sysconf(_SC_PAGESIZE) : 4096;
    const uintptr_t lo = (uintptr_t)base & ~(uintptr_t)(pg - 1);
    madvise((void *)lo, (uintptr_t)base + len - lo, MADV_WILLNEED);
    const volatile uint8_t *p = (const volatile uint8_t *)base;
    for (size_t i = 0; i < len; i += (size_t)pg) (void)p[i];
    (void)p[len - 1];
}

Q35_API void q35_plat_mmap_prefetch(Q35PlatMmap *m)
{
    if (!m || !m->base) return;
    q35_plat_prefetch(m->base, m->len);
    if (!preload_enabled()) return;
    const uint8_t *b = (const uint8_t *)m->base;
    uint64_t hlen = 0;  /* a safetensors shard: 8-byte header length, then a JSON object */
    if (m->len < 10) return;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
    if (hlen > m->len - 8 || b[8] != '{') return;
    preload_fn preload = (preload_fn)q35cuda_sym("q35cu_preload_safetensors");
    if (preload) preload(m->base, m->len);  /* a failure leaves first-touch uploads in place */
}

Q35_API uint64_t q35_plat_avail_phys(void)
{
    FILE *f = fopen("/proc/meminfo", "r");
    if (f) {
        char line[256];
        unsigned long long kb = 0;
        int found = 0;
        while (fgets(line, sizeof line, f))
            if (sscanf(line, "MemAvailable: %llu kB", &kb) == 1) {
                found = 1;
                break;
            }
        fclose(f);
        if (found) return (uint64_t)kb * 1024u;
    }
    const long pages = sysconf(_SC_AVPHYS_PAGES), pg = sysconf(_SC_PAGESIZE);
    return (pages > 0 && pg > 0) ? (uint64_t)pages * (uint64_t)pg : 0;
}

Q35_API size_t q35_plat_peak_rss(void)
{
    struct rusage ru;
    if (getrusage(RUSAGE_SELF, &ru) != 0 || ru.ru_maxrss <= 0) return 0;
    return (size_t)ru.ru_maxrss * 1024u;  /* Linux reports kilobytes */
}

static long read_long(const char *path)
{
    FILE *f = fopen(path, "r");
    if (!f) return -1;
    long v = -1;
    if (fscanf(f, "%ld", &v) != 1) v = -1;
    fclose(f);
    return v;
}

Q35_API int q35_plat_num_phys_cores(void)
{
    cpu_set_t set;
    CPU_ZERO(&set);
    const int have_mask = sched_getaffinity(0, sizeof set, &set) == 0;
    enum { kMax = 4096 };
    long seen[kMax];
    int n = 0, usable = 0;
    for (int cpu = 0; cpu < CPU_SETSIZE && cpu < kMax; ++cpu) {
        if (have_mask && !CPU_ISSET(cpu, &set)) continue;
        char path[128];
        snprintf(path, sizeof path, "/sys/devices/system/cpu/cpu%d/topology/core_id", cpu);
        const long core = read_long(path);
        snprintf(path, sizeof path, "/sys/devices/system/cpu/cpu%d/topology/physical_package_id", cpu);
        const long pkg = read_long(path);
        if (core < 0 || pkg < 0) continue;
        ++usable;
        const long key = pkg * 65536 + core;
        int dup = 0;
        for (int i = 0; i < n; ++i)
            if (seen[i] == key) {
                dup = 1;
                break;
            }
        if (!dup && n < kMax) seen[n++] = key;
    }
    if (n > 0 && usable > 0) return n;
    const long online = sysconf(_SC_NPROCESSORS_ONLN);
    return online > 0 ? (int)online : 0;
}

Q35_API char *q35_plat_strdup(const char *s) { return s ? strdup(s) : NULL; }

Q35_API int q35_plat_path_join(char *dst, size_t cap, const char *dir, const char *name)
{
    if (!dst || !cap || !dir || !name) return -1;
    const int n = snprintf(dst, cap, "%s/%s", dir, name);
    return (n >= 0 && (size_t)n < cap) ? 0 : -1;
}

Q35_API int q35_plat_sock_init(void) { return 0; }

Q35_API int q35_plat_sock_listen(int port)
{
    const int fd = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) return -1;
    const int one = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
    struct sockaddr_in a;
    memset(&a, 0, sizeof a);
    a.sin_family = AF_INET;
    a.sin_addr.s_addr = htonl(INADDR_LOOPBACK);
    a.sin_port = htons((uint16_t)port);
    if (bind(fd, (struct sockaddr *)&a, sizeof a) != 0 || listen(fd, 16) != 0) {
        close(fd);
        return -1;
    }
    return fd;
}

Q35_API int q35_plat_sock_accept(int lfd)
{
    for (;;) {
        const int fd = accept4(lfd, NULL, NULL, SOCK_CLOEXEC);
        if (fd < 0 && errno == EINTR) continue;
        return fd;
    }
}

Q35_API int q35_plat_sock_recv(int fd, void *buf, size_t len)
{
    for (;;) {
        const ssize_t r = recv(fd, buf, len, 0);
        if (r < 0 && errno == EINTR) continue;
        return (int)r;
    }
}

Q35_API int q35_plat_sock_send(int fd, const void *buf, size_t len)
{
    for (;;) {
        const ssize_t r = send(fd, buf, len, MSG_NOSIGNAL);
        if (r < 0 && errno == EINTR) continue;
        return (int)r;
    }
}

Q35_API void q35_plat_sock_close(int fd)
{
    if (fd >= 0) close(fd);
}
