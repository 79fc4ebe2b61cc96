/* Expert reads from a checkpoint file: the reference engine's demand reader as a host component.
 *
 * Replaces read_range / read_pieces (stbl/model.cu:269-308) and the reader set-up (stbl/model.cu:978-987):
 * a set of host threads reads byte ranges of the checkpoint in 2 MiB pieces with pread, through an
 * O_DIRECT descriptor where the file system takes it (buffered reads otherwise), into caller-owned
 * memory.  The expert cache's file-backed mode (stbl_cache_create_file, include/stbl_moe.h) reads the
 * missing experts of each call with it into page-locked staging; it is exported on its own for callers
 * that stage experts themselves and for the host-side tests.  No CUDA calls: usable without a GPU.
 *
 * Differences from the reference: the threads are started once (the reference starts them per call),
 * every range is read as its 4096-byte aligned superset in both modes (so the data of a range sits at
 * the same place whichever mode reads it), a read refused with EINVAL by an O_DIRECT descriptor (or a
 * short read that leaves an unaligned remainder) is retried buffered instead of failing, EINTR is
 * retried, and a failure reports which range, offset and errno. */
#ifndef STBL_IO_H
#define STBL_IO_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct stbl_reader stbl_reader;

/* Opens `path` with `threads` reader threads (0: 4, the reference's STBL_READ_THREADS default; at most
 * 64).  direct = 1: O_DIRECT where the file system takes it (an open refused falls back to buffered
 * reads, as the reference does), 0: buffered.  0 and *out on success; -1 and a message in err. */
int stbl_reader_open(const char *path, int threads, int direct, stbl_reader **out, char *err, int errlen);

/* Bytes a destination region must hold for a range of `bytes` bytes: the 4096-byte aligned superset. */
uint64_t stbl_reader_region_bytes(uint64_t bytes);

/* Reads n ranges (file offset off[i], length bytes[i]) into region[i] (4096-byte aligned, at least
 * stbl_reader_region_bytes(bytes[i]) bytes) with all reader threads, 2 MiB per piece; the data of range
 * i starts at region[i] + at[i] (at[i] = off[i] mod 4096).  Blocks until every piece is in.  0 on
 * success; -1 when an argument is bad, a read failed or the file ended inside a range (message in
 * stbl_reader_error).  One call at a time per reader. */
int stbl_reader_read(stbl_reader *r, int n, const uint64_t *off, const uint64_t *bytes, void *const *region,
                     uint64_t *at);

/* Counters since open: pieces read, bytes read (aligned supersets), seconds spent in stbl_reader_read,
 * and *direct = 1 while reads go through O_DIRECT. */
int stbl_reader_stats(const stbl_reader *r, uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct);

/* Host-side fault injection for tests: counting from this call, piece read number `after` (0: the next
 * one) and every later one fail with errno err_no, as a pread error would.  err_no 0 switches it off. */
int stbl_reader_inject_error(stbl_reader *r, int64_t after, int err_no);

/* The message of the last failure ("" when none). */
const char *stbl_reader_error(const stbl_reader *r);
void stbl_reader_close(stbl_reader *r);

#ifdef __cplusplus
}
#endif

#endif
