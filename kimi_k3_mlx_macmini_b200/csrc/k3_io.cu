// Checkpoint byte ranges -> host or device memory (host code only).
//
// The reference reads one MXFP4 projection as ONE contiguous read: in its checkpoints a
// projection's `weight_scale` tensor starts where its `weight_packed` tensor ends, so
// the pair is fetched together and sliced (air_llm/models/kimi_k3/loader.py:229-266,
// `_read_pair`); byte ranges come from the manifest records (offset, nbytes;
// tools/k3_manifest.py:97-156). Here the same reads are plain POSIX `pread`s:
//
//   * k3_file_read_ranges: n (offset, nbytes, dst) ranges of one file. Ranges adjacent
//     in the file AND in memory merge into one read (the packed + scale pair); the
//     merged reads are cut into pieces of at most 8 MiB and spread over `threads`
//     threads, each looping until its piece is complete (pread may return short).
//   * k3_file_read_to_device: the same ranges into device memory through a caller-owned
//     pinned staging buffer used as two halves: the disk read of one half overlaps the
//     host->device copy (cudaMemcpyAsync on `stream`) of the other.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "k3_common.cuh"

namespace k3 {
namespace {

constexpr int64_t kIoPiece = int64_t(8) << 20;   // bytes per read task

struct Task {
    int64_t off;
    int64_t n;
    uint8_t* dst;
};

struct Fd {
    int fd = -1;
    ~Fd() {
        if (fd >= 0) ::close(fd);
    }
};

// Merges adjacent ranges (file and memory both contiguous) and cuts the result into
// read tasks of at most kIoPiece bytes.
std::vector<Task> plan_reads(const int64_t* off, const int64_t* nb, int n, uint8_t* const* dst) {
    std::vector<Task> merged;
    for (int i = 0; i < n; ++i) {
        if (nb[i] == 0) continue;
        if (!merged.empty()) {
            Task& t = merged.back();
            if (t.off + t.n == off[i] && t.dst + t.n == dst[i]) {
                t.n += nb[i];
                continue;
            }
        }
        merged.push_back({off[i], nb[i], dst[i]});
    }
    std::vector<Task> tasks;
    for (const Task& t : merged)
        for (int64_t o = 0; o < t.n; o += kIoPiece)
            tasks.push_back({t.off + o, std::min(kIoPiece, t.n - o), t.dst + o});
    return tasks;
}

// Runs the tasks on `threads` threads; returns 0 or the first errno / -1 on EOF.
int run_reads(int fd, const std::vector<Task>& tasks, int threads) {
    std::atomic<size_t> next{0};
    std::atomic<int> err{0};
    auto worker = [&]() {
        for (;;) {
            const size_t i = next.fetch_add(1);
            if (i >= tasks.size() || err.load()) return;
            const Task& t = tasks[i];
            int64_t done = 0;
            while (done < t.n) {
                const ssize_t r = ::pread(fd, t.dst + done, size_t(t.n - done), off_t(t.off + done));
                if (r < 0) {
                    if (errno == EINTR) continue;
                    int z = 0;
                    err.compare_exchange_strong(z, errno);
                    return;
                }
                if (r == 0) {                                   // past the end of the file
                    int z = 0;
                    err.compare_exchange_strong(z, -1);
                    return;
                }
                done += r;
            }
        }
    };
    const int nt = std::max(1, std::min<int>(threads, int(tasks.size())));
    std::vector<std::thread> pool;
    for (int i = 1; i < nt; ++i) pool.emplace_back(worker);
    worker();
    for (auto& th : pool) th.join();
    return err.load();
}

int open_checked(const char* path, Fd& f, const char* who) {
    if (!path) return fail(K3_ERR_INVALID, std::string(who) + ": path is NULL");
    f.fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (f.fd < 0) return fail(K3_ERR_IO, std::string(who) + ": cannot open " + path + ": " + std::strerror(errno));
    return K3_OK;
}

int check_ranges(int fd, const int64_t* off, const int64_t* nb, int n, const char* who) {
    if (n < 0 || (n > 0 && (!off || !nb))) return fail(K3_ERR_INVALID, std::string(who) + ": bad range arrays");
    struct stat st {};
    if (::fstat(fd, &st) != 0) return fail(K3_ERR_IO, std::string(who) + ": fstat failed");
    for (int i = 0; i < n; ++i)
        if (off[i] < 0 || nb[i] < 0 || off[i] + nb[i] > int64_t(st.st_size))
            return fail(K3_ERR_INVALID, std::string(who) + ": range " + std::to_string(i) + " [" +
                                            std::to_string(off[i]) + ", +" + std::to_string(nb[i]) +
                                            ") lies outside the file (" + std::to_string(st.st_size) + " bytes)");
    return K3_OK;
}

int io_error(int e, const char* who) {
    return fail(K3_ERR_IO, std::string(who) + (e < 0 ? ": unexpected end of file" : ": read failed: ") +
                               (e < 0 ? "" : std::strerror(e)));
}

}  // namespace
}  // namespace k3

using namespace k3;

extern "C" K3_API int k3_file_read_ranges(const char* path, const int64_t* offsets, const int64_t* nbytes, int n,
                                          void* const* dst, int threads, int64_t* bytes_read_out) {
    Fd f;
    if (int rc = open_checked(path, f, "k3_file_read_ranges")) return rc;
    if (int rc = check_ranges(f.fd, offsets, nbytes, n, "k3_file_read_ranges")) return rc;
    if (n > 0 && !dst) return fail(K3_ERR_INVALID, "k3_file_read_ranges: dst is NULL");
    for (int i = 0; i < n; ++i)
        if (nbytes[i] > 0 && !dst[i]) return fail(K3_ERR_INVALID, "k3_file_read_ranges: NULL destination");
    const auto tasks = plan_reads(offsets, nbytes, n, reinterpret_cast<uint8_t* const*>(dst));
    if (int e = run_reads(f.fd, tasks, threads)) return io_error(e, "k3_file_read_ranges");
    if (bytes_read_out) {
        int64_t t = 0;
        for (int i = 0; i < n; ++i) t += nbytes[i];
        *bytes_read_out = t;
    }
    return K3_OK;
}

extern "C" K3_API int k3_file_read_to_device(const char* path, const int64_t* offsets, const int64_t* nbytes, int n,
                                             void* const* device_dst, void* pinned_staging, size_t staging_bytes,
                                             int threads, void* stream) {
    Fd f;
    if (int rc = open_checked(path, f, "k3_file_read_to_device")) return rc;
    if (int rc = check_ranges(f.fd, offsets, nbytes, n, "k3_file_read_to_device")) return rc;
    if (!pinned_staging || staging_bytes < 2 * 4096)
        return fail(K3_ERR_INVALID, "k3_file_read_to_device: staging buffer missing or under 8 KiB");
    if (n > 0 && !device_dst) return fail(K3_ERR_INVALID, "k3_file_read_to_device: device_dst is NULL");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t half = int64_t(staging_bytes / 2) & ~int64_t(4095);
    uint8_t* stage[2] = {static_cast<uint8_t*>(pinned_staging), static_cast<uint8_t*>(pinned_staging) + half};
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (auto& e : done)
        if (int rc = cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate")) return rc;
    int rc = K3_OK;
    bool used[2] = {false, false};
    int h = 0;
    // walk the ranges in pieces of at most one half
    for (int i = 0; i < n && rc == K3_OK; ++i) {
        if (nbytes[i] > 0 && !device_dst[i]) {
            rc = fail(K3_ERR_INVALID, "k3_file_read_to_device: NULL destination");
            break;
        }
        for (int64_t o = 0; o < nbytes[i] && rc == K3_OK; o += half) {
            const int64_t len = std::min(half, nbytes[i] - o);
            if (used[h] && (rc = cuda_check(cudaEventSynchronize(done[h]), "cudaEventSynchronize"))) break;
            const int64_t off = offsets[i] + o;
            uint8_t* const dst[1] = {stage[h]};
            const auto tasks = plan_reads(&off, &len, 1, dst);
            if (int e = run_reads(f.fd, tasks, threads)) {
                rc = io_error(e, "k3_file_read_to_device");
                break;
            }
            if ((rc = cuda_check(cudaMemcpyAsync(static_cast<uint8_t*>(device_dst[i]) + o, stage[h], size_t(len),
                                                 cudaMemcpyHostToDevice, s),
                                 "cudaMemcpyAsync")))
                break;
            if ((rc = cuda_check(cudaEventRecord(done[h], s), "cudaEventRecord"))) break;
            used[h] = true;
            h ^= 1;
        }
    }
    // the staging buffer belongs to the caller again only after its copies finished
    for (int j = 0; j < 2; ++j)
        if (used[j]) {
            const int r2 = cuda_check(cudaEventSynchronize(done[j]), "cudaEventSynchronize");
            if (rc == K3_OK) rc = r2;
        }
    for (auto& e : done) cudaEventDestroy(e);
    return rc;
}
