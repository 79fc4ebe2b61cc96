// Checkpoint reader (include/stbl_io.h), the reference's read_range / read_pieces (stbl/model.cu:269-308)
// with its O_DIRECT set-up (stbl/model.cu:978-987), as a pool of host threads started once.
//
// A call turns each range into its 4096-byte aligned superset [off & ~4095, roundup(off + bytes, 4096))
// and cuts that into 2 MiB pieces; the threads (and the calling thread) take pieces from a shared
// counter until none are left or one has failed.  A piece may end past the end of the file (the
// aligned tail of the last tensor): only the bytes up to the range's end must arrive.
#include "../../include/stbl_io.h"
#include "reader.cuh"

#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <stdexcept>

namespace stbl {

ExpertReader::ExpertReader(const char *path, int threads, bool direct) {
    fd_ = open(path, O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) throw std::runtime_error(std::string("cannot open ") + path + ": " + strerror(errno));
    if (direct) {
        fd_direct_ = open(path, O_RDONLY | O_CLOEXEC | O_DIRECT);  // -1 where the file system refuses it
        direct_on_ = fd_direct_ >= 0;
    }
    const int n = threads > 0 ? std::min(threads, 64) : 4;
    for (int i = 1; i < n; i++) threads_.emplace_back(&ExpertReader::worker, this);
}

ExpertReader::~ExpertReader() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto &t : threads_) t.join();
    if (fd_direct_ >= 0) close(fd_direct_);
    if (fd_ >= 0) close(fd_);
}

void ExpertReader::fail(const std::string &m) {
    std::lock_guard<std::mutex> lk(err_mu_);
    if (ok_.exchange(false)) err_ = m;
}

std::string ExpertReader::error() const {
    std::lock_guard<std::mutex> lk(err_mu_);
    return err_;
}

void ExpertReader::stats(uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct) const {
    if (pieces) *pieces = pieces_.load();
    if (bytes) *bytes = bytes_.load();
    if (seconds) *seconds = 1e-9 * (double)ns_.load();
    if (direct) *direct = direct_on_.load() ? 1 : 0;
}

void ExpertReader::inject_error(int64_t after, int err_no) {
    inject_errno_ = err_no;
    inject_left_ = err_no ? after : -1;
}

bool ExpertReader::read_piece(const Piece &p) {
    uint64_t got = 0;
    while (got < p.need) {
        // O_DIRECT needs an aligned offset, length and buffer: after an unaligned short read the rest
        // of the piece is read buffered
        const bool dir = direct_on_.load() && got % kReadAlign == 0;
        ssize_t n;
        int e = 0;
        const int64_t left = inject_left_.load();
        if (inject_errno_.load() && left >= 0 && inject_left_.fetch_sub(1) <= 0) {
            inject_left_ = 0;
            n = -1, e = inject_errno_.load();
        } else {
            n = pread(dir ? fd_direct_ : fd_, p.dst + got, p.len - got, (off_t)(p.start + got));
            e = n < 0 ? errno : 0;
        }
        if (n < 0) {
            if (e == EINTR) continue;
            if (e == EINVAL && dir) {
                direct_on_ = false;  // the file system takes O_DIRECT opens but not its reads
                continue;
            }
            fail("read of range " + std::to_string(p.range) + " at offset " + std::to_string(p.start + got) +
                 " failed: " + strerror(e));
            return false;
        }
        if (n == 0) {
            fail("file ends at offset " + std::to_string(p.start + got) + " inside range " + std::to_string(p.range));
            return false;
        }
        got += (uint64_t)n;
    }
    pieces_++;
    bytes_ += got;
    return true;
}

void ExpertReader::drain() {
    for (size_t j; ok_.load() && (j = next_++) < batch_.size();) read_piece(batch_[j]);
}

void ExpertReader::worker() {
    uint64_t seen = 0;
    for (;;) {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        active_++;
        lk.unlock();
        drain();
        lk.lock();
        if (--active_ == 0) cv_done_.notify_all();
    }
}

bool ExpertReader::read(int n, const uint64_t *off, const uint64_t *bytes, uint8_t *const *region, uint64_t *at) {
    std::lock_guard<std::mutex> call(call_mu_);
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<Piece> ps;
    for (int i = 0; i < n; i++) {
        if (((uintptr_t)region[i] & (kReadAlign - 1)) != 0) {
            std::lock_guard<std::mutex> lk(err_mu_);
            err_ = "region " + std::to_string(i) + " is not 4096-byte aligned";
            return false;
        }
        const uint64_t a0 = off[i] & ~(kReadAlign - 1), end = off[i] + bytes[i];
        const uint64_t a1 = (end + kReadAlign - 1) & ~(kReadAlign - 1);
        at[i] = off[i] - a0;
        for (uint64_t s = a0; s < a1 && bytes[i] > 0; s += kReadPiece) {
            const uint64_t e = std::min(a1, s + kReadPiece);
            ps.push_back(Piece{s, e - s, std::min(e, end) - s, region[i] + (s - a0), i});
        }
    }
    {
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return active_ == 0; });  // threads still leaving the previous batch
        batch_ = std::move(ps);
        next_ = 0;
        ok_ = true;
        gen_++;
    }
    cv_.notify_all();
    drain();
    {
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return active_ == 0; });
    }
    ns_ += (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
    return ok_.load();
}

}  // namespace stbl

struct stbl_reader {
    stbl::ExpertReader *r = nullptr;
    std::string err;
};

namespace {
int fail_msg(char *err, int errlen, const std::string &m) {
    if (err && errlen > 0) {
        const size_t n = std::min((size_t)errlen - 1, m.size());
        m.copy(err, n);
        err[n] = 0;
    }
    return -1;
}
}  // namespace

extern "C" {

int stbl_reader_open(const char *path, int threads, int direct, stbl_reader **out, char *err, int errlen) {
    if (!path || !out) return fail_msg(err, errlen, "null argument");
    if (threads < 0) return fail_msg(err, errlen, "threads must be >= 0");
    try {
        auto *h = new stbl_reader();
        h->r = new stbl::ExpertReader(path, threads, direct != 0);
        *out = h;
        return 0;
    } catch (const std::exception &e) {
        return fail_msg(err, errlen, e.what());
    }
}

uint64_t stbl_reader_region_bytes(uint64_t bytes) { return stbl::read_region_bytes(bytes); }

int stbl_reader_read(stbl_reader *r, int n, const uint64_t *off, const uint64_t *bytes, void *const *region, uint64_t *at) {
    if (!r) return -1;
    if (n < 0 || (n > 0 && (!off || !bytes || !region || !at))) {
        r->err = "bad arguments";
        return -1;
    }
    std::vector<uint8_t *> dst(n);
    for (int i = 0; i < n; i++) dst[i] = static_cast<uint8_t *>(region[i]);
    if (!r->r->read(n, off, bytes, dst.data(), at)) {
        r->err = r->r->error();
        return -1;
    }
    return 0;
}

int stbl_reader_stats(const stbl_reader *r, uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct) {
    if (!r) return -1;
    r->r->stats(pieces, bytes, seconds, direct);
    return 0;
}

int stbl_reader_inject_error(stbl_reader *r, int64_t after, int err_no) {
    if (!r || after < 0 || err_no < 0) return -1;
    r->r->inject_error(after, err_no);
    return 0;
}

const char *stbl_reader_error(const stbl_reader *r) { return r ? r->err.c_str() : "null reader"; }

void stbl_reader_close(stbl_reader *r) {
    if (!r) return;
    delete r->r;
    delete r;
}

}  // extern "C"
