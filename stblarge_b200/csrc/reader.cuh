// Checkpoint reader (include/stbl_io.h): host threads reading byte ranges of a file with pread in
// 2 MiB pieces, O_DIRECT where the file system takes it.  Shared by the C ABI in reader.cu and the
// expert cache's file-backed mode in cache.cu.  Host code only.
#pragma once

#include <stdint.h>

#include <atomic>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace stbl {

constexpr uint64_t kReadPiece = 2ull << 20;  // bytes per pread (stbl/model.cu:269)
constexpr uint64_t kReadAlign = 4096;        // O_DIRECT alignment of offsets, lengths and buffers

inline uint64_t read_region_bytes(uint64_t bytes) {
    return ((bytes + kReadAlign - 1) & ~(kReadAlign - 1)) + kReadAlign;
}

class ExpertReader {
  public:
    // throws std::runtime_error when the file cannot be opened
    ExpertReader(const char *path, int threads, bool direct);
    ~ExpertReader();
    ExpertReader(const ExpertReader &) = delete;
    ExpertReader &operator=(const ExpertReader &) = delete;

    // range i -> region[i] (4096-aligned, read_region_bytes(bytes[i]) long), data at region[i] + at[i];
    // false on failure (error() says why).  One call at a time.
    bool read(int n, const uint64_t *off, const uint64_t *bytes, uint8_t *const *region, uint64_t *at);
    std::string error() const;
    void stats(uint64_t *pieces, uint64_t *bytes, double *seconds, int *direct) const;
    void inject_error(int64_t after, int err_no);

  private:
    struct Piece {
        uint64_t start, len, need;  // aligned file offset, bytes to request, bytes that must arrive
        uint8_t *dst;
        int range;
    };
    void worker();
    void drain();
    bool read_piece(const Piece &p);
    void fail(const std::string &m);

    int fd_ = -1, fd_direct_ = -1;
    std::atomic<bool> direct_on_{false};
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_, cv_done_;
    uint64_t gen_ = 0;
    bool stop_ = false;
    int active_ = 0;
    std::vector<Piece> batch_;
    std::atomic<size_t> next_{0};
    std::atomic<bool> ok_{true};
    std::atomic<uint64_t> pieces_{0}, bytes_{0};
    std::atomic<uint64_t> ns_{0};  // time spent in read(); stats() may run during a read
    std::atomic<int64_t> inject_left_{-1};
    std::atomic<int> inject_errno_{0};
    mutable std::mutex err_mu_;
    std::string err_;
    std::mutex call_mu_;
};

}  // namespace stbl
