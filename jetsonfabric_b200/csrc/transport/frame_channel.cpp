// In-box frame channel: one request/reply mailbox pair in POSIX shared memory
// between a stage server process and the processes that call it.
//
// The reference moves each stage operation as one Stagewire v2 frame over a
// keep-alive HTTP connection (runtime/transport/http_stage_transport.cpp:
// 481-599): a POST whose body is the frame, answered by a status line and a
// response frame. Between processes on one box the same exchange needs no
// socket, no HTTP framing and no copy through the kernel: the caller writes
// the request frame (metadata prefix and payload, two pieces, as the
// reference's EncodedStageFrameView holds them) straight into the shared
// segment, the server reads it in place and writes its reply frame and status
// into the second mailbox. Frames are opaque bytes here; the codec is the
// caller's.
//
// Layout: a 4 KiB header, then the request mailbox, then the reply mailbox,
// each `capacity` bytes (the segment is sparse: pages are touched only as far
// as frames reach). Hand-off is one 32-bit state word (idle -> request ->
// reply -> idle) waited on with process-shared futexes; every wait is bounded
// and returns JFB_STATUS_TIMEOUT. One caller at a time holds the channel (a
// lock word in the header, also waited on with a bound); a caller that gave up
// waiting leaves its request behind, and the next caller discards that
// request's late reply by its sequence number. A lock whose holder process has
// exited is taken over, and so is the name of a server that exited without
// closing its channel.
#include "jfb/jfb_stagewire.h"

#include <linux/futex.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <fcntl.h>
#include <signal.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kMagic = 0x4A464348u;  // "JFCH"
constexpr uint32_t kVersion = 2;
constexpr uint64_t kHeaderBytes = 4096;
constexpr uint64_t kDefaultCapacity = (512ull << 20) + (1ull << 20) + 4096;  // max payload + max metadata + header

enum : uint32_t { kIdle = 0, kRequest = 1, kReply = 2, kClosed = 3 };

struct alignas(64) Header {
    alignas(4) uint32_t magic;  // written last by the server, through std::atomic_ref
    uint32_t version;
    uint64_t capacity;
    alignas(64) std::atomic<uint32_t> state;
    alignas(64) std::atomic<uint32_t> caller;  // 0 = free, else the holder's pid
    std::atomic<uint32_t> server_pid;          // the creating process, for stale-name takeover
    alignas(64) uint64_t request_seq;
    uint64_t request_bytes;
    uint64_t reply_seq;
    uint64_t reply_bytes;
    int32_t reply_status;
    uint32_t reply_is_frame;
};
static_assert(sizeof(Header) <= kHeaderBytes, "channel header must fit its page");
static_assert(sizeof(std::atomic<uint32_t>) == sizeof(uint32_t), "futex word must be a plain 32-bit word");

jfb_status ok() {
    jfb_status s;
    s.code = JFB_STATUS_OK;
    s.message[0] = '\0';
    return s;
}

jfb_status fail(jfb_status_code code, const char * fmt, ...) {
    jfb_status s;
    s.code = code;
    va_list a;
    va_start(a, fmt);
    std::vsnprintf(s.message, sizeof(s.message), fmt, a);
    va_end(a);
    return s;
}

using Clock = std::chrono::steady_clock;

void futex_wake(std::atomic<uint32_t> * word) {
    syscall(SYS_futex, reinterpret_cast<uint32_t *>(word), FUTEX_WAKE, INT32_MAX, nullptr, nullptr, 0);
}

// Waits until `word` leaves `seen` or the deadline passes (spurious returns are fine).
void futex_wait(std::atomic<uint32_t> * word, uint32_t seen, Clock::time_point deadline) {
    const auto left = deadline - Clock::now();
    if (left <= Clock::duration::zero()) return;
    const auto ns = std::chrono::duration_cast<std::chrono::nanoseconds>(left).count();
    timespec ts;
    ts.tv_sec = static_cast<time_t>(ns / 1000000000);
    ts.tv_nsec = static_cast<long>(ns % 1000000000);
    syscall(SYS_futex, reinterpret_cast<uint32_t *>(word), FUTEX_WAIT, seen, &ts, nullptr, 0);
}

std::string shm_name(const char * name) { return std::string("/jfb-stage-") + name; }

// A process that no longer exists (it cannot answer or release anything).
bool process_gone(uint32_t pid) { return pid != 0 && kill(static_cast<pid_t>(pid), 0) != 0 && errno == ESRCH; }

// An existing segment named `path` whose creating server has exited without
// closing it: removes the name so that a new server can take it.
bool unlink_if_stale(const std::string & path) {
    const int fd = shm_open(path.c_str(), O_RDWR, 0);
    if (fd < 0) return errno == ENOENT;
    struct stat st;
    bool stale = false;
    if (fstat(fd, &st) == 0 && static_cast<uint64_t>(st.st_size) >= kHeaderBytes) {
        void * p = mmap(nullptr, kHeaderBytes, PROT_READ, MAP_SHARED, fd, 0);
        if (p != MAP_FAILED) {
            const auto * h = static_cast<const Header *>(p);
            stale = process_gone(h->server_pid.load(std::memory_order_acquire));
            munmap(p, kHeaderBytes);
        }
    }
    close(fd);
    if (stale) shm_unlink(path.c_str());
    return stale;
}

bool valid_name(const char * name) {
    if (name == nullptr || name[0] == '\0' || std::strlen(name) > 200) return false;
    for (const char * p = name; *p; ++p) {
        const char c = *p;
        if (!((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '-' || c == '_' ||
              c == '.')) {
            return false;
        }
    }
    return true;
}

}  // namespace

struct jfb_frame_channel {
    Header * header = nullptr;
    uint8_t * base = nullptr;
    uint64_t mapped = 0;
    bool server = false;
    std::string name;
    uint64_t seq = 0;                 // caller: last request sequence sent
    std::vector<uint8_t> reply_copy;  // caller: the last reply, valid until the next call

    uint8_t * request_area() const { return base + kHeaderBytes; }
    uint8_t * reply_area() const { return base + kHeaderBytes + header->capacity; }

    ~jfb_frame_channel() {
        if (base != nullptr) {
            if (server) {
                header->state.store(kClosed, std::memory_order_release);
                futex_wake(&header->state);
            }
            munmap(base, mapped);
        }
        if (server) shm_unlink(shm_name(name.c_str()).c_str());
    }
};

extern "C" jfb_status jfb_frame_channel_create(const char * name, uint64_t capacity, jfb_frame_channel ** out) {
    if (out == nullptr || !valid_name(name)) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "channel names are 1-200 characters of [A-Za-z0-9._-]");
    }
    *out = nullptr;
    if (capacity == 0) capacity = kDefaultCapacity;
    capacity = (capacity + 4095) / 4096 * 4096;
    const std::string path = shm_name(name);
    int fd = shm_open(path.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
    int err = fd < 0 ? errno : 0;
    if (fd < 0 && err == EEXIST && unlink_if_stale(path)) {
        fd = shm_open(path.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
        err = fd < 0 ? errno : 0;
    }
    if (fd < 0) {
        return fail(err == EEXIST ? JFB_STATUS_INVALID_ARGUMENT : JFB_STATUS_IO_ERROR,
                    "could not create stage channel %s: %s", name, std::strerror(err));
    }
    const uint64_t bytes = kHeaderBytes + 2 * capacity;
    if (ftruncate(fd, static_cast<off_t>(bytes)) != 0) {
        const int e = errno;
        close(fd);
        shm_unlink(path.c_str());
        return fail(JFB_STATUS_IO_ERROR, "could not size stage channel %s: %s", name, std::strerror(e));
    }
    void * p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) {
        shm_unlink(path.c_str());
        return fail(JFB_STATUS_IO_ERROR, "could not map stage channel %s", name);
    }
    auto * ch = new (std::nothrow) jfb_frame_channel();
    if (ch == nullptr) {
        munmap(p, bytes);
        shm_unlink(path.c_str());
        return fail(JFB_STATUS_OUT_OF_MEMORY, "out of host memory");
    }
    ch->base = static_cast<uint8_t *>(p);
    ch->mapped = bytes;
    ch->server = true;
    ch->name = name;
    ch->header = new (ch->base) Header();
    ch->header->capacity = capacity;
    ch->header->version = kVersion;
    ch->header->state.store(kIdle, std::memory_order_relaxed);
    ch->header->caller.store(0, std::memory_order_relaxed);
    ch->header->server_pid.store(static_cast<uint32_t>(getpid()), std::memory_order_relaxed);
    std::atomic_thread_fence(std::memory_order_release);
    std::atomic_ref<uint32_t>(ch->header->magic).store(kMagic, std::memory_order_release);
    *out = ch;
    return ok();
}

extern "C" jfb_status jfb_frame_channel_open(const char * name, uint32_t timeout_ms, jfb_frame_channel ** out) {
    if (out == nullptr || !valid_name(name)) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "channel names are 1-200 characters of [A-Za-z0-9._-]");
    }
    *out = nullptr;
    const std::string path = shm_name(name);
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    int fd = -1;
    for (;;) {
        fd = shm_open(path.c_str(), O_RDWR, 0);
        if (fd >= 0) {
            struct stat st;
            if (fstat(fd, &st) == 0 && static_cast<uint64_t>(st.st_size) > kHeaderBytes) {
                void * p = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
                close(fd);
                fd = -1;
                if (p == MAP_FAILED) return fail(JFB_STATUS_IO_ERROR, "could not map stage channel %s", name);
                auto * h = static_cast<Header *>(p);
                const uint32_t magic =
                    std::atomic_ref<uint32_t>(h->magic).load(std::memory_order_acquire);
                if (magic == kMagic && h->version == kVersion &&
                    kHeaderBytes + 2 * h->capacity == static_cast<uint64_t>(st.st_size)) {
                    auto * ch = new (std::nothrow) jfb_frame_channel();
                    if (ch == nullptr) {
                        munmap(p, static_cast<size_t>(st.st_size));
                        return fail(JFB_STATUS_OUT_OF_MEMORY, "out of host memory");
                    }
                    ch->base = static_cast<uint8_t *>(p);
                    ch->mapped = static_cast<uint64_t>(st.st_size);
                    ch->header = h;
                    ch->name = name;
                    ch->seq = h->request_seq;
                    *out = ch;
                    return ok();
                }
                munmap(p, static_cast<size_t>(st.st_size));
            } else {
                close(fd);
            }
        }
        if (Clock::now() >= deadline) {
            return fail(JFB_STATUS_NOT_FOUND, "stage channel %s has no server", name);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
}

extern "C" uint64_t jfb_frame_channel_capacity(const jfb_frame_channel * ch) {
    return ch == nullptr ? 0 : ch->header->capacity;
}

extern "C" jfb_status jfb_frame_channel_call(jfb_frame_channel * ch, const void * head, uint64_t head_bytes,
                                             const void * body, uint64_t body_bytes, uint32_t timeout_ms,
                                             int32_t * status, int32_t * is_frame, const uint8_t ** reply,
                                             uint64_t * reply_bytes) {
    if (ch == nullptr || ch->server || status == nullptr || is_frame == nullptr || reply == nullptr ||
        reply_bytes == nullptr || (head_bytes > 0 && head == nullptr) || (body_bytes > 0 && body == nullptr)) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "frame channel call needs an opened channel and output slots");
    }
    Header * h = ch->header;
    if (head_bytes > h->capacity || body_bytes > h->capacity - head_bytes) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "frame of %llu bytes exceeds the channel's %llu",
                    static_cast<unsigned long long>(head_bytes + body_bytes),
                    static_cast<unsigned long long>(h->capacity));
    }
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    const uint32_t me = static_cast<uint32_t>(getpid());
    // the channel's caller lock; a holder that has exited is replaced
    for (;;) {
        uint32_t holder = 0;
        if (h->caller.compare_exchange_strong(holder, me, std::memory_order_acquire)) break;
        if (process_gone(holder) && h->caller.compare_exchange_strong(holder, me, std::memory_order_acquire)) break;
        if (Clock::now() >= deadline) return fail(JFB_STATUS_TIMEOUT, "stage channel %s is busy", ch->name.c_str());
        futex_wait(&h->caller, holder, std::min(deadline, Clock::now() + std::chrono::milliseconds(2)));
    }
    const auto release = [&] {
        h->caller.store(0, std::memory_order_release);
        futex_wake(&h->caller);
    };
    // an earlier caller's abandoned request: wait for its reply and drop it
    for (;;) {
        const uint32_t s = h->state.load(std::memory_order_acquire);
        if (s == kIdle) break;
        if (s == kClosed) {
            release();
            return fail(JFB_STATUS_EXECUTION_FAILED, "stage channel %s was closed by its server", ch->name.c_str());
        }
        if (s == kReply) {
            h->state.store(kIdle, std::memory_order_release);
            break;
        }
        if (Clock::now() >= deadline) {
            release();
            return fail(JFB_STATUS_TIMEOUT, "stage channel %s: the previous request is still running",
                        ch->name.c_str());
        }
        futex_wait(&h->state, s, deadline);
    }
    uint8_t * dst = ch->request_area();
    if (head_bytes) std::memcpy(dst, head, head_bytes);
    if (body_bytes) std::memcpy(dst + head_bytes, body, body_bytes);
    const uint64_t seq = h->request_seq + 1;
    h->request_seq = seq;
    h->request_bytes = head_bytes + body_bytes;
    ch->seq = seq;
    h->state.store(kRequest, std::memory_order_release);
    futex_wake(&h->state);
    for (;;) {
        const uint32_t s = h->state.load(std::memory_order_acquire);
        if (s == kReply && h->reply_seq == seq) break;
        if (s == kClosed) {
            release();
            return fail(JFB_STATUS_EXECUTION_FAILED, "stage channel %s was closed by its server", ch->name.c_str());
        }
        if (Clock::now() >= deadline) {
            release();
            return fail(JFB_STATUS_TIMEOUT, "stage channel %s: no reply within %u ms", ch->name.c_str(), timeout_ms);
        }
        futex_wait(&h->state, s, deadline);
    }
    const uint64_t n = h->reply_bytes;
    if (n > h->capacity) {
        h->state.store(kIdle, std::memory_order_release);
        release();
        return fail(JFB_STATUS_FORMAT_ERROR, "stage channel %s: reply length out of range", ch->name.c_str());
    }
    ch->reply_copy.assign(ch->reply_area(), ch->reply_area() + n);
    *status = h->reply_status;
    *is_frame = static_cast<int32_t>(h->reply_is_frame);
    h->state.store(kIdle, std::memory_order_release);
    futex_wake(&h->state);
    release();
    *reply = ch->reply_copy.data();
    *reply_bytes = n;
    return ok();
}

extern "C" jfb_status jfb_frame_channel_receive(jfb_frame_channel * ch, uint32_t timeout_ms, const uint8_t ** frame,
                                                uint64_t * frame_bytes) {
    if (ch == nullptr || !ch->server || frame == nullptr || frame_bytes == nullptr) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "frame channel receive needs a created channel and output slots");
    }
    Header * h = ch->header;
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        const uint32_t s = h->state.load(std::memory_order_acquire);
        if (s == kRequest) break;
        if (Clock::now() >= deadline) return fail(JFB_STATUS_TIMEOUT, "no request within %u ms", timeout_ms);
        futex_wait(&h->state, s, deadline);
    }
    if (h->request_bytes > h->capacity) return fail(JFB_STATUS_FORMAT_ERROR, "request length out of range");
    *frame = ch->request_area();
    *frame_bytes = h->request_bytes;
    return ok();
}

extern "C" jfb_status jfb_frame_channel_reply(jfb_frame_channel * ch, int32_t status, int32_t is_frame,
                                              const void * head, uint64_t head_bytes, const void * body,
                                              uint64_t body_bytes) {
    if (ch == nullptr || !ch->server || (head_bytes > 0 && head == nullptr) || (body_bytes > 0 && body == nullptr)) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "frame channel reply needs a created channel");
    }
    Header * h = ch->header;
    if (h->state.load(std::memory_order_acquire) != kRequest) {
        return fail(JFB_STATUS_INVALID_ARGUMENT, "frame channel reply without a pending request");
    }
    uint64_t total = head_bytes + body_bytes;
    if (head_bytes > h->capacity || body_bytes > h->capacity - head_bytes) {
        // too large for the mailbox: answer with an error the caller can read
        static const char kTooLarge[] =
            "{\"error\":\"runtime_stage_reply_too_large\",\"message\":\"stage reply exceeds the channel capacity\"}";
        head = kTooLarge;
        head_bytes = sizeof(kTooLarge) - 1;
        body_bytes = 0;
        total = head_bytes;
        status = 502;
        is_frame = 0;
    }
    uint8_t * dst = ch->reply_area();
    if (head_bytes) std::memcpy(dst, head, head_bytes);
    if (body_bytes) std::memcpy(dst + head_bytes, body, body_bytes);
    h->reply_bytes = total;
    h->reply_status = status;
    h->reply_is_frame = is_frame ? 1u : 0u;
    h->reply_seq = h->request_seq;
    h->state.store(kReply, std::memory_order_release);
    futex_wake(&h->state);
    return ok();
}

extern "C" void jfb_frame_channel_close(jfb_frame_channel * ch) { delete ch; }
