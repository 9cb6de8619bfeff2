/* The engine's platform abstraction layer, as the unchanged qwen35-c sources
 * call it (interface of qwen35-c/src/q35_plat.h:1-74; the reference ships
 * only a Windows implementation, qwen35-c/src/q35_plat_win.c, whose
 * directory walk and read-only mapping are stubs elsewhere).
 *
 * libq35plat.so (qwen38-in-c_b200/pal/q35_plat_posix.c) implements every
 * entry point with POSIX/Linux calls, so the engine -- loader, layers,
 * tokenizer, CLI -- builds and loads a model on the Linux B200 host next to
 * libq35cuda.so.  The declarations below are the reference's, unchanged. */
#ifndef Q35_PLAT_H
#define Q35_PLAT_H

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

/* whole file into a NUL-terminated heap buffer (free with q35_plat_free);
 * NULL on any failure, *out_len untouched then */
void *q35_plat_read_file(const char *path, size_t *out_len);

/* alignment: a power of two >= sizeof(void *) */
void *q35_plat_aligned_alloc(size_t alignment, size_t size);
void q35_plat_aligned_free(void *p);

/* a large-page mapping for big buffers, or NULL (the caller then uses its
 * own allocator); q35_plat_large_free releases only what this returned */
void *q35_plat_large_alloc(size_t size);
void q35_plat_large_free(void *p);

void q35_plat_free(void *p);

/* monotonic seconds */
double q35_plat_now(void);

/* regular files of a directory (no ".", "..", subdirectories); a returned
 * name stays valid until the next call on the same handle */
typedef struct Q35PlatDir Q35PlatDir;
Q35PlatDir *q35_plat_dir_open(const char *dir);
const char *q35_plat_dir_next(Q35PlatDir *d);
void q35_plat_dir_close(Q35PlatDir *d);

int q35_plat_fseek64(FILE *f, int64_t offset, int whence);
int64_t q35_plat_ftell64(FILE *f);

/* read-only mapping of a whole file; NULL on failure (an empty file too) */
typedef struct Q35PlatMmap Q35PlatMmap;
Q35PlatMmap *q35_plat_mmap_ro(const char *path, const uint8_t **out_base);
void q35_plat_munmap(Q35PlatMmap *m);
void q35_plat_mmap_prefetch(Q35PlatMmap *m);

/* bytes, 0 = unknown */
uint64_t q35_plat_avail_phys(void);
size_t q35_plat_peak_rss(void);

/* physical cores (SMT siblings counted once), <= 0 = unknown */
int q35_plat_num_phys_cores(void);

char *q35_plat_strdup(const char *s);

/* dst = dir "/" name; 0, or -1 when it does not fit in cap */
int q35_plat_path_join(char *dst, size_t cap, const char *dir, const char *name);

/* page in [base, base + len) ahead of use; no-op on NULL / 0 */
void q35_plat_prefetch(const void *base, size_t len);

/* loopback TCP server sockets */
int q35_plat_sock_init(void);
int q35_plat_sock_listen(int port);
int q35_plat_sock_accept(int lfd);
int q35_plat_sock_recv(int fd, void *buf, size_t len);
int q35_plat_sock_send(int fd, const void *buf, size_t len);
void q35_plat_sock_close(int fd);

#ifdef __cplusplus
}
#endif

#endif
