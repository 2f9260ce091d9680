/*
 * JFM v2 package reader (C11, libc + pthreads only).
 *
 * Implements the jf_* ABI of include/jetsonfabric/engine.h from the published
 * package description (reference docs/jfm-v2-format.md). Behaviour that callers
 * and tests depend on follows the reference loader
 * (runtime/engines/native/src/engine.c):
 *   - segment selection for a stage plan (engine.c:181-196, 641-643): metadata
 *     and shared segments always, input only when layer_start == 0, layer
 *     segments inside [layer_start, layer_end), output only on the last stage;
 *   - manifest topology checks and their status codes (engine.c:513-640);
 *   - tensor-record validation (engine.c:330-470) and name uniqueness
 *     (engine.c:497-511);
 *   - SHA-256 verification of every selected segment file when
 *     plan->verify_hashes is set (engine.c:262-276).
 *
 * Layout of the implementation: the manifest is parsed into a small table
 * first, every check that needs no file I/O runs before anything is mapped,
 * and only then are the selected segment files opened, mapped and indexed.
 */
#define _GNU_SOURCE
#include "jetsonfabric/engine.h"

#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

enum {
    MANIFEST_HEADER_BYTES = 64,
    MANIFEST_RECORD_BYTES = 72,
    SEGMENT_HEADER_BYTES = 64,
    TENSOR_RECORD_BYTES = 80,
    PAYLOAD_ALIGNMENT = 64,
    FORMAT_VERSION = 2,
};

#define MAX_MANIFEST_BYTES (16u * 1024u * 1024u)
#define MAX_LAYER_COUNT 4096u
#define MAX_TENSOR_COUNT 1000000u

enum segment_kind {
    SEGMENT_SHARED = 0,
    SEGMENT_INPUT = 1,
    SEGMENT_LAYER = 2,
    SEGMENT_OUTPUT = 3,
    SEGMENT_METADATA = 4,
};

static const char manifest_magic[8] = {'J', 'F', 'M', 'O', 'D', 'E', 'L', '2'};
static const char segment_magic[8] = {'J', 'F', 'S', 'E', 'G', 'M', '0', '2'};

typedef struct segment_entry {
    uint32_t kind;
    int32_t layer;
    uint64_t tensor_count;
    uint64_t payload_bytes;
    uint64_t file_bytes;
    uint8_t digest[32];
    const char * path;
    uint32_t path_length;
    int selected;
} segment_entry;

typedef struct mapped_file {
    void * base;
    size_t bytes;
} mapped_file;

struct jf_model {
    mapped_file * files;
    size_t file_count;
    jf_tensor_view * tensors;
    size_t tensor_count;
    const void * metadata;
    size_t metadata_bytes;
    uint8_t source_digest[32];
    jf_model_stats stats;
};

/* ---- little helpers -------------------------------------------------- */

static jf_status ok_status(void) {
    jf_status status;
    status.code = JF_STATUS_OK;
    status.message[0] = '\0';
    return status;
}

static jf_status fail(jf_status_code code, const char * format, ...) {
    jf_status status;
    status.code = code;
    va_list args;
    va_start(args, format);
    (void) vsnprintf(status.message, sizeof(status.message), format, args);
    va_end(args);
    return status;
}

static uint32_t le32(const uint8_t * p) {
    return (uint32_t) p[0] | ((uint32_t) p[1] << 8) | ((uint32_t) p[2] << 16) |
        ((uint32_t) p[3] << 24);
}

static uint64_t le64(const uint8_t * p) {
    return (uint64_t) le32(p) | ((uint64_t) le32(p + 4) << 32);
}

/* offset + length <= limit, without overflow */
static int within(uint64_t offset, uint64_t length, uint64_t limit) {
    return offset <= limit && length <= limit - offset;
}

static int checked_add(uint64_t a, uint64_t b, uint64_t * out) {
    if (a > UINT64_MAX - b) return 0;
    *out = a + b;
    return 1;
}

static int checked_mul(uint64_t a, uint64_t b, uint64_t * out) {
    if (a != 0 && b > UINT64_MAX / a) return 0;
    *out = a * b;
    return 1;
}

static int all_zero(const uint8_t * p, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        if (p[i] != 0) return 0;
    }
    return 1;
}

static int compare_bytes(const char * a, size_t an, const char * b, size_t bn) {
    const int c = memcmp(a, b, an < bn ? an : bn);
    if (c != 0) return c;
    return (an > bn) - (an < bn);
}

/* Segment paths are single, non-hidden file names inside the package. */
static int path_is_safe(const char * path, uint32_t length) {
    if (length == 0 || length > 255 || path[0] == '.') return 0;
    for (uint32_t i = 0; i < length; ++i) {
        if (path[i] == '/' || path[i] == '\\' || path[i] == '\0') return 0;
    }
    return 1;
}

/* ---- storage geometry ------------------------------------------------- */

typedef struct type_geometry {
    uint16_t elements;
    uint16_t bytes;
} type_geometry;

/* Canonical (elements, bytes) per storage block, indexed by JFM type id; the
 * table in the format description's "Stable Tensor Types" section. */
static const type_geometry geometry_table[36] = {
    {0, 0},     {1, 4},     {1, 2},     {32, 18},   {32, 20},   {32, 22},
    {32, 24},   {32, 34},   {32, 36},   {256, 84},  {256, 110}, {256, 144},
    {256, 176}, {256, 210}, {256, 292}, {256, 66},  {256, 74},  {256, 98},
    {256, 50},  {32, 18},   {256, 110}, {256, 82},  {256, 136}, {1, 1},
    {1, 2},     {1, 4},     {1, 8},     {1, 8},     {256, 56},  {1, 2},
    {256, 54},  {256, 66},  {32, 17},   {64, 36},   {128, 18},  {64, 18},
};

jf_status jf_tensor_type_layout(uint32_t type, uint32_t * block_elements, uint32_t * block_bytes) {
    if (block_elements == NULL || block_bytes == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "tensor layout outputs are required");
    }
    if (type == 0 || type >= sizeof(geometry_table) / sizeof(geometry_table[0])) {
        return fail(JF_STATUS_FORMAT_ERROR, "unsupported JFM tensor type %u", type);
    }
    *block_elements = geometry_table[type].elements;
    *block_bytes = geometry_table[type].bytes;
    return ok_status();
}

/* ---- manifest ----------------------------------------------------------- */

static jf_status slurp_manifest(int dir, uint8_t ** bytes_out, size_t * size_out) {
    const int fd = openat(dir, "manifest.jfm", O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
    if (fd < 0) return fail(JF_STATUS_IO_ERROR, "open manifest.jfm: %s", strerror(errno));
    struct stat info;
    if (fstat(fd, &info) != 0) {
        const int e = errno;
        close(fd);
        return fail(JF_STATUS_IO_ERROR, "stat manifest.jfm: %s", strerror(e));
    }
    if (!S_ISREG(info.st_mode) || info.st_size < 0 ||
        (uint64_t) info.st_size > MAX_MANIFEST_BYTES) {
        close(fd);
        return fail(JF_STATUS_FORMAT_ERROR, "manifest.jfm is not a bounded regular file");
    }
    const size_t size = (size_t) info.st_size;
    uint8_t * bytes = malloc(size > 0 ? size : 1);
    if (bytes == NULL) {
        close(fd);
        return fail(JF_STATUS_OUT_OF_MEMORY, "allocate %zu manifest bytes", size);
    }
    size_t done = 0;
    while (done < size) {
        const ssize_t got = read(fd, bytes + done, size - done);
        if (got < 0 && errno == EINTR) continue;
        if (got <= 0) {
            const int e = got < 0 ? errno : EIO;
            free(bytes);
            close(fd);
            return fail(JF_STATUS_IO_ERROR, "read manifest.jfm: %s", strerror(e));
        }
        done += (size_t) got;
    }
    close(fd);
    *bytes_out = bytes;
    *size_out = size;
    return ok_status();
}

static int wanted_by_plan(const segment_entry * s, uint32_t start, uint32_t end, uint32_t layers) {
    switch (s->kind) {
    case SEGMENT_METADATA:
    case SEGMENT_SHARED:
        return 1;
    case SEGMENT_INPUT:
        return start == 0;
    case SEGMENT_OUTPUT:
        return end == layers;
    case SEGMENT_LAYER:
        return s->layer >= 0 && (uint32_t) s->layer >= start && (uint32_t) s->layer < end;
    default:
        return 0;
    }
}

static int compare_segment_path(const void * a, const void * b) {
    const segment_entry * x = a;
    const segment_entry * y = b;
    return compare_bytes(x->path, x->path_length, y->path, y->path_length);
}

/* ---- segment files ------------------------------------------------------ */

static jf_status map_segment_file(int dir, const segment_entry * s, int verify, int evict,
                                  mapped_file * out) {
    char name[256];
    memcpy(name, s->path, s->path_length);
    name[s->path_length] = '\0';
    const int fd = openat(dir, name, O_RDONLY | O_CLOEXEC | O_NOFOLLOW);
    if (fd < 0) return fail(JF_STATUS_IO_ERROR, "open %s: %s", name, strerror(errno));
    struct stat info;
    if (fstat(fd, &info) != 0) {
        const int e = errno;
        close(fd);
        return fail(JF_STATUS_IO_ERROR, "stat %s: %s", name, strerror(e));
    }
    if (!S_ISREG(info.st_mode) || info.st_size <= 0 ||
        (uint64_t) info.st_size != s->file_bytes || s->file_bytes > SIZE_MAX) {
        close(fd);
        return fail(JF_STATUS_FORMAT_ERROR, "%s size or file type does not match manifest", name);
    }
    if (evict) {
#ifdef POSIX_FADV_DONTNEED
        const int advice = posix_fadvise(fd, 0, 0, POSIX_FADV_DONTNEED);
        if (advice != 0) {
            close(fd);
            return fail(JF_STATUS_IO_ERROR, "evict %s from page cache: %s", name, strerror(advice));
        }
#else
        close(fd);
        return fail(JF_STATUS_IO_ERROR, "page-cache eviction is unsupported");
#endif
    }
    void * base = mmap(NULL, (size_t) info.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    const int map_errno = errno;
    close(fd);
    if (base == MAP_FAILED) return fail(JF_STATUS_IO_ERROR, "map %s: %s", name, strerror(map_errno));
    out->base = base;
    out->bytes = (size_t) info.st_size;
    (void) verify;  /* digests are checked afterwards, in parallel */
    return ok_status();
}

/* ---- parallel digest verification --------------------------------------- */

typedef struct verify_job {
    const segment_entry ** segments;
    const mapped_file * files;
    size_t count;
    atomic_size_t next;
    atomic_int first_bad;  /* index of a mismatching file, or -1 */
} verify_job;

static void * verify_worker(void * arg) {
    verify_job * job = arg;
    for (;;) {
        const size_t i = atomic_fetch_add(&job->next, 1);
        if (i >= job->count) return NULL;
        uint8_t digest[32];
        jf_sha256_buffer(job->files[i].base, job->files[i].bytes, digest);
        if (memcmp(digest, job->segments[i]->digest, 32) != 0) {
            int expected = -1;
            (void) atomic_compare_exchange_strong(&job->first_bad, &expected, (int) i);
        }
    }
}

/* Verifies every mapped segment against its manifest digest using up to one
 * thread per file (bounded by the online CPU count). */
static jf_status verify_digests(const segment_entry ** segments, const mapped_file * files, size_t count) {
    verify_job job;
    job.segments = segments;
    job.files = files;
    job.count = count;
    atomic_init(&job.next, 0);
    atomic_init(&job.first_bad, -1);
    long cpus = sysconf(_SC_NPROCESSORS_ONLN);
    if (cpus < 1) cpus = 1;
    size_t workers = count < (size_t) cpus ? count : (size_t) cpus;
    if (workers > 64) workers = 64;
    pthread_t threads[64];
    size_t started = 0;
    for (; started + 1 < workers; ++started) {
        if (pthread_create(&threads[started], NULL, verify_worker, &job) != 0) break;
    }
    (void) verify_worker(&job);
    for (size_t i = 0; i < started; ++i) pthread_join(threads[i], NULL);
    const int bad = atomic_load(&job.first_bad);
    if (bad >= 0) {
        return fail(JF_STATUS_FORMAT_ERROR, "%.*s checksum does not match manifest",
                    (int) segments[bad]->path_length, segments[bad]->path);
    }
    return ok_status();
}

/* Parses one tensor segment's index into model->tensors[*next ...]. */
static jf_status index_tensor_segment(const segment_entry * s, const mapped_file * file,
                                      jf_model * model, size_t * next) {
    const uint8_t * base = file->base;
    const uint64_t size = file->bytes;
    if (size < SEGMENT_HEADER_BYTES) return fail(JF_STATUS_FORMAT_ERROR, "tensor segment is truncated");
    if (memcmp(base, segment_magic, 8) != 0 || le32(base + 8) != FORMAT_VERSION ||
        !all_zero(base + 32, SEGMENT_HEADER_BYTES - 32)) {
        return fail(JF_STATUS_FORMAT_ERROR, "tensor segment has an unsupported header");
    }
    const uint32_t count = le32(base + 12);
    const uint64_t index_bytes = le64(base + 16);
    const uint64_t payload_total = le64(base + 24);
    if (count != s->tensor_count || payload_total != s->payload_bytes ||
        !within(SEGMENT_HEADER_BYTES, index_bytes, size)) {
        return fail(JF_STATUS_FORMAT_ERROR, "tensor segment has an invalid index");
    }
    const uint64_t index_end = SEGMENT_HEADER_BYTES + index_bytes;
    if (index_end > UINT64_MAX - PAYLOAD_ALIGNMENT) {
        return fail(JF_STATUS_FORMAT_ERROR, "tensor segment index overflows");
    }
    const uint64_t payload_start = (index_end + PAYLOAD_ALIGNMENT - 1) / PAYLOAD_ALIGNMENT * PAYLOAD_ALIGNMENT;
    if (payload_start > size) {
        return fail(JF_STATUS_FORMAT_ERROR, "tensor segment data starts past end of file");
    }

    uint64_t cursor = SEGMENT_HEADER_BYTES;
    uint64_t last_end = payload_start;
    uint64_t seen_payload = 0;
    for (uint32_t t = 0; t < count; ++t) {
        if (!within(cursor, TENSOR_RECORD_BYTES, index_end)) {
            return fail(JF_STATUS_FORMAT_ERROR, "tensor record is truncated");
        }
        const uint8_t * r = base + cursor;
        const uint32_t type = le32(r);
        const uint32_t rank = le32(r + 4);
        const int32_t layer = (int32_t) le32(r + 8);
        const uint32_t flags = le32(r + 12);
        const uint64_t offset = le64(r + 48);
        const uint64_t length = le64(r + 56);
        const uint32_t name_length = le32(r + 64);
        const uint32_t block_elements = le32(r + 68);
        const uint32_t block_bytes = le32(r + 72);
        const uint32_t reserved = le32(r + 76);
        cursor += TENSOR_RECORD_BYTES;

        uint32_t canon_elements = 0, canon_bytes = 0;
        const int known = jf_tensor_type_layout(type, &canon_elements, &canon_bytes).code == JF_STATUS_OK;
        if (!known || block_elements != canon_elements || block_bytes != canon_bytes ||
            flags != 0 || reserved != 0 || rank == 0 || rank > 4 || name_length == 0 ||
            name_length > 1024 || !within(cursor, name_length, index_end) ||
            offset % PAYLOAD_ALIGNMENT != 0 || offset < last_end || !within(offset, length, size)) {
            return fail(JF_STATUS_FORMAT_ERROR, "tensor segment contains an invalid record");
        }
        const int layer_ok = s->kind == SEGMENT_LAYER ? layer == s->layer : layer == -1;
        if (!layer_ok) return fail(JF_STATUS_FORMAT_ERROR, "tensor layer does not match its segment");
        if (*next >= model->tensor_count) {
            return fail(JF_STATUS_FORMAT_ERROR, "segment declares too many tensors");
        }
        uint64_t shape[4];
        uint64_t rows = 1;
        for (uint32_t d = 0; d < 4; ++d) {
            shape[d] = le64(r + 16 + 8 * d);
            if (shape[d] == 0 || (d >= rank && shape[d] != 1)) {
                return fail(JF_STATUS_FORMAT_ERROR, "tensor shape is invalid");
            }
            if (d > 0 && !checked_mul(rows, shape[d], &rows)) {
                return fail(JF_STATUS_FORMAT_ERROR, "tensor shape overflows");
            }
        }
        uint64_t row_bytes = 0, expected = 0;
        if (shape[0] % block_elements != 0 ||
            !checked_mul(shape[0] / block_elements, block_bytes, &row_bytes) ||
            !checked_mul(row_bytes, rows, &expected) || expected != length ||
            !checked_add(offset, length, &last_end) ||
            !checked_add(seen_payload, length, &seen_payload)) {
            return fail(JF_STATUS_FORMAT_ERROR, "tensor storage size is inconsistent");
        }
        jf_tensor_view * v = &model->tensors[(*next)++];
        v->name = (const char *) base + cursor;
        v->name_length = name_length;
        v->type = type;
        v->rank = rank;
        v->storage_block_elements = block_elements;
        v->storage_block_bytes = block_bytes;
        memcpy(v->shape, shape, sizeof(shape));
        v->layer = layer;
        v->data = base + offset;
        v->size = length;
        cursor += name_length;
        cursor = (cursor + 7u) & ~(uint64_t) 7u;
    }
    if (cursor != index_end || seen_payload != s->payload_bytes) {
        return fail(JF_STATUS_FORMAT_ERROR, "tensor index or payload total does not match manifest");
    }
#ifdef MADV_SEQUENTIAL
    (void) madvise(file->base, file->bytes, MADV_SEQUENTIAL);
#endif
    return ok_status();
}

static int compare_tensor_name(const void * a, const void * b) {
    const jf_tensor_view * x = a;
    const jf_tensor_view * y = b;
    return compare_bytes(x->name, x->name_length, y->name, y->name_length);
}

static void release(jf_model * model) {
    if (model == NULL) return;
    for (size_t i = 0; i < model->file_count; ++i) {
        if (model->files[i].base != NULL) munmap(model->files[i].base, model->files[i].bytes);
    }
    free(model->files);
    free(model->tensors);
    free(model);
}

/* Reads the manifest table and applies every check that needs no segment I/O. */
static jf_status parse_manifest(const uint8_t * m, size_t size, const jf_stage_plan * requested,
                                segment_entry ** table_out, uint32_t * count_out,
                                jf_stage_plan * plan_out, jf_model_stats * stats) {
    if (size < MANIFEST_HEADER_BYTES || memcmp(m, manifest_magic, 8) != 0 ||
        le32(m + 8) != FORMAT_VERSION || le32(m + 60) != 0) {
        return fail(JF_STATUS_FORMAT_ERROR, "manifest has an unsupported header");
    }
    const uint32_t layers = le32(m + 12);
    const uint64_t source_bytes = le64(m + 16);
    const uint32_t count = le32(m + 56);
    jf_stage_plan plan = *requested;
    if (plan.layer_end == JF_ALL_LAYERS) plan.layer_end = layers;
    if (layers == 0 || layers > MAX_LAYER_COUNT || source_bytes == 0 ||
        plan.layer_start >= plan.layer_end || plan.layer_end > layers) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "stage range or model dimensions are invalid");
    }
    if (count < layers + 3u || count > layers + 4u) {
        return fail(JF_STATUS_FORMAT_ERROR, "manifest segment topology is invalid");
    }
    segment_entry * table = calloc(count, sizeof(*table));
    uint8_t * layer_seen = calloc(layers, 1);
    if (table == NULL || layer_seen == NULL) {
        free(table);
        free(layer_seen);
        return fail(JF_STATUS_OUT_OF_MEMORY, "allocate manifest topology index");
    }
    jf_status status = ok_status();
    uint32_t kind_count[5] = {0, 0, 0, 0, 0};
    uint64_t cursor = MANIFEST_HEADER_BYTES;
    memset(stats, 0, sizeof(*stats));
    for (uint32_t i = 0; i < count && status.code == JF_STATUS_OK; ++i) {
        if (!within(cursor, MANIFEST_RECORD_BYTES, size)) {
            status = fail(JF_STATUS_FORMAT_ERROR, "manifest segment index is truncated");
            break;
        }
        const uint8_t * r = m + cursor;
        segment_entry * s = &table[i];
        s->kind = le32(r);
        s->layer = (int32_t) le32(r + 4);
        s->tensor_count = le64(r + 8);
        s->payload_bytes = le64(r + 16);
        s->file_bytes = le64(r + 24);
        memcpy(s->digest, r + 32, 32);
        s->path_length = le32(r + 64);
        const uint32_t reserved = le32(r + 68);
        cursor += MANIFEST_RECORD_BYTES;
        s->path = (const char *) m + cursor;
        const int record_ok = within(cursor, s->path_length, size) &&
            path_is_safe(s->path, s->path_length) && s->file_bytes != 0 &&
            s->kind <= SEGMENT_METADATA && reserved == 0 &&
            (s->kind == SEGMENT_METADATA || (s->tensor_count != 0 && s->payload_bytes != 0));
        if (!record_ok) {
            status = fail(JF_STATUS_FORMAT_ERROR, "manifest contains an invalid segment");
            break;
        }
        cursor += s->path_length;
        if (s->kind == SEGMENT_LAYER) {
            if (s->layer < 0 || (uint32_t) s->layer >= layers || layer_seen[s->layer]) {
                status = fail(JF_STATUS_FORMAT_ERROR, "manifest layer topology is invalid");
                break;
            }
            layer_seen[s->layer] = 1;
        } else if (s->layer != -1) {
            status = fail(JF_STATUS_FORMAT_ERROR, "global segment declares a layer");
            break;
        } else if (s->kind == SEGMENT_METADATA && (s->tensor_count != 0 || s->payload_bytes != 0)) {
            status = fail(JF_STATUS_FORMAT_ERROR, "metadata segment declares tensors");
            break;
        }
        ++kind_count[s->kind];
        if (!checked_add(stats->total_tensor_count, s->tensor_count, &stats->total_tensor_count) ||
            !checked_add(stats->total_weight_bytes, s->payload_bytes, &stats->total_weight_bytes) ||
            stats->total_tensor_count > MAX_TENSOR_COUNT) {
            status = fail(JF_STATUS_FORMAT_ERROR, "manifest tensor totals overflow");
            break;
        }
        s->selected = wanted_by_plan(s, plan.layer_start, plan.layer_end, layers);
        if (s->selected &&
            (!checked_add(stats->selected_tensor_count, s->tensor_count, &stats->selected_tensor_count) ||
             !checked_add(stats->selected_weight_bytes, s->payload_bytes, &stats->selected_weight_bytes) ||
             !checked_add(stats->mapped_bytes, s->file_bytes, &stats->mapped_bytes))) {
            status = fail(JF_STATUS_FORMAT_ERROR, "selected model totals overflow");
            break;
        }
    }
    if (status.code == JF_STATUS_OK &&
        (cursor != size || kind_count[SEGMENT_METADATA] != 1 || kind_count[SEGMENT_SHARED] > 1 ||
         kind_count[SEGMENT_INPUT] != 1 || kind_count[SEGMENT_OUTPUT] != 1)) {
        status = fail(JF_STATUS_FORMAT_ERROR, "manifest does not define one complete model");
    }
    for (uint32_t l = 0; status.code == JF_STATUS_OK && l < layers; ++l) {
        if (!layer_seen[l]) status = fail(JF_STATUS_FORMAT_ERROR, "manifest is missing a model layer");
    }
    if (status.code == JF_STATUS_OK) {
        segment_entry * sorted = malloc(count * sizeof(*sorted));
        if (sorted == NULL) {
            status = fail(JF_STATUS_OUT_OF_MEMORY, "allocate manifest path index");
        } else {
            memcpy(sorted, table, count * sizeof(*sorted));
            qsort(sorted, count, sizeof(*sorted), compare_segment_path);
            for (uint32_t i = 1; i < count; ++i) {
                if (compare_segment_path(&sorted[i - 1], &sorted[i]) == 0) {
                    status = fail(JF_STATUS_FORMAT_ERROR, "manifest contains duplicate segment paths");
                    break;
                }
            }
            free(sorted);
        }
    }
    if (status.code == JF_STATUS_OK &&
        (stats->selected_tensor_count > SIZE_MAX || stats->mapped_bytes > SIZE_MAX)) {
        status = fail(JF_STATUS_FORMAT_ERROR, "selected model exceeds addressable memory");
    }
    free(layer_seen);
    if (status.code != JF_STATUS_OK) {
        free(table);
        return status;
    }
    stats->layer_start = plan.layer_start;
    stats->layer_end = plan.layer_end;
    stats->layer_count = layers;
    *table_out = table;
    *count_out = count;
    *plan_out = plan;
    return ok_status();
}

jf_status jf_model_open(const char * package_path, const jf_stage_plan * plan, jf_model ** output) {
    if (package_path == NULL || package_path[0] == '\0' || plan == NULL || output == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "package path, plan, and output are required");
    }
    *output = NULL;
    const int dir = open(package_path, O_RDONLY | O_DIRECTORY | O_CLOEXEC | O_NOFOLLOW);
    if (dir < 0) return fail(JF_STATUS_IO_ERROR, "open package %s: %s", package_path, strerror(errno));

    uint8_t * manifest = NULL;
    size_t manifest_size = 0;
    jf_status status = slurp_manifest(dir, &manifest, &manifest_size);
    segment_entry * table = NULL;
    uint32_t segment_count = 0;
    jf_stage_plan resolved;
    jf_model_stats stats;
    if (status.code == JF_STATUS_OK) {
        status = parse_manifest(manifest, manifest_size, plan, &table, &segment_count, &resolved, &stats);
    }
    jf_model * model = NULL;
    if (status.code == JF_STATUS_OK) {
        model = calloc(1, sizeof(*model));
        size_t selected_files = 0;
        for (uint32_t i = 0; i < segment_count; ++i) selected_files += table[i].selected ? 1u : 0u;
        if (model != NULL) {
            model->files = calloc(selected_files > 0 ? selected_files : 1, sizeof(*model->files));
            model->tensor_count = (size_t) stats.selected_tensor_count;
            model->tensors = calloc(model->tensor_count > 0 ? model->tensor_count : 1, sizeof(*model->tensors));
        }
        if (model == NULL || model->files == NULL || model->tensors == NULL) {
            release(model);
            model = NULL;
            status = fail(JF_STATUS_OUT_OF_MEMORY, "allocate selected model index");
        }
    }
    if (status.code == JF_STATUS_OK) {
        memcpy(model->source_digest, manifest + 24, 32);
        model->stats = stats;
        size_t next_tensor = 0;
        const segment_entry ** mapped_segments = calloc(segment_count, sizeof(*mapped_segments));
        if (mapped_segments == NULL) status = fail(JF_STATUS_OUT_OF_MEMORY, "allocate segment map");
        for (uint32_t i = 0; i < segment_count && status.code == JF_STATUS_OK; ++i) {
            const segment_entry * s = &table[i];
            if (!s->selected) continue;
            mapped_file * file = &model->files[model->file_count];
            status = map_segment_file(dir, s, resolved.verify_hashes != 0,
                                      resolved.evict_before_open != 0, file);
            if (file->base != NULL) mapped_segments[model->file_count++] = s;
        }
        if (status.code == JF_STATUS_OK && resolved.verify_hashes != 0) {
            status = verify_digests(mapped_segments, model->files, model->file_count);
        }
        for (size_t f = 0; f < model->file_count && status.code == JF_STATUS_OK; ++f) {
            const segment_entry * s = mapped_segments[f];
            mapped_file * file = &model->files[f];
            if (s->kind == SEGMENT_METADATA) {
                if (file->bytes < 4 || memcmp(file->base, "GGUF", 4) != 0) {
                    status = fail(JF_STATUS_FORMAT_ERROR, "metadata segment is not a GGUF header");
                } else {
                    model->metadata = file->base;
                    model->metadata_bytes = file->bytes;
                }
            } else {
                status = index_tensor_segment(s, file, model, &next_tensor);
            }
        }
        free(mapped_segments);
        if (status.code == JF_STATUS_OK) {
            int unique = next_tensor == model->tensor_count;
            if (unique) {
                qsort(model->tensors, model->tensor_count, sizeof(*model->tensors), compare_tensor_name);
                for (size_t i = 1; i < model->tensor_count && unique; ++i) {
                    unique = compare_tensor_name(&model->tensors[i - 1], &model->tensors[i]) != 0;
                }
            }
            if (!unique) {
                status = fail(JF_STATUS_FORMAT_ERROR, "selected tensor index is incomplete or ambiguous");
            }
        }
        if (status.code != JF_STATUS_OK) {
            release(model);
            model = NULL;
        }
    }
    free(table);
    free(manifest);
    close(dir);
    if (status.code == JF_STATUS_OK) *output = model;
    return status;
}

void jf_model_close(jf_model * model) { release(model); }

jf_model_stats jf_model_get_stats(const jf_model * model) {
    jf_model_stats empty;
    memset(&empty, 0, sizeof(empty));
    return model == NULL ? empty : model->stats;
}

size_t jf_model_tensor_count(const jf_model * model) { return model == NULL ? 0 : model->tensor_count; }

jf_status jf_model_tensor_at(const jf_model * model, size_t index, jf_tensor_view * tensor) {
    if (model == NULL || tensor == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "model and tensor output are required");
    }
    if (index >= model->tensor_count) {
        return fail(JF_STATUS_NOT_FOUND, "tensor index %zu is out of range", index);
    }
    *tensor = model->tensors[index];
    return ok_status();
}

jf_status jf_model_find_tensor(const jf_model * model, const char * name, jf_tensor_view * tensor) {
    if (model == NULL || name == NULL || name[0] == '\0' || tensor == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "model, tensor name, and output are required");
    }
    /* tensors are sorted by name after open: binary search */
    const size_t length = strlen(name);
    size_t lo = 0, hi = model->tensor_count;
    while (lo < hi) {
        const size_t mid = lo + (hi - lo) / 2;
        const jf_tensor_view * v = &model->tensors[mid];
        const int c = compare_bytes(v->name, v->name_length, name, length);
        if (c == 0) {
            *tensor = *v;
            return ok_status();
        }
        if (c < 0) lo = mid + 1; else hi = mid;
    }
    return fail(JF_STATUS_NOT_FOUND, "tensor %s is not selected", name);
}

jf_status jf_model_get_source_sha256(const jf_model * model, uint8_t digest[32]) {
    if (model == NULL || digest == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "model and digest output are required");
    }
    memcpy(digest, model->source_digest, 32);
    return ok_status();
}

jf_status jf_model_get_gguf_metadata(const jf_model * model, const void ** data, size_t * size) {
    if (model == NULL || data == NULL || size == NULL) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "model, metadata data, and size are required");
    }
    *data = model->metadata;
    *size = model->metadata_bytes;
    return ok_status();
}

/* ---- prefetch ----------------------------------------------------------- */

typedef struct prefetch_job {
    const jf_model * model;
    size_t page;
    atomic_size_t next_file;
    uint64_t * file_sums;
} prefetch_job;

/* FNV-1a (64-bit) over one byte per page and the last byte: enough to force
 * every page in without the scan being optimised away. */
static void * prefetch_worker(void * arg) {
    prefetch_job * job = arg;
    for (;;) {
        const size_t f = atomic_fetch_add(&job->next_file, 1);
        if (f >= job->model->file_count) return NULL;
        const mapped_file * file = &job->model->files[f];
#ifdef MADV_WILLNEED
        (void) madvise(file->base, file->bytes, MADV_WILLNEED);
#endif
        const volatile uint8_t * bytes = file->base;
        uint64_t h = 0xcbf29ce484222325ull;
        for (size_t off = 0; off < file->bytes; off += job->page) h = (h ^ bytes[off]) * 0x100000001b3ull;
        h = (h ^ bytes[file->bytes - 1]) * 0x100000001b3ull;
        job->file_sums[f] = h;
    }
}

jf_status jf_model_prefetch_parallel(jf_model * model, uint32_t thread_count, uint64_t * checksum) {
    if (model == NULL || thread_count == 0 || thread_count > 256) {
        return fail(JF_STATUS_INVALID_ARGUMENT, "model and 1-256 prefetch threads are required");
    }
    const long page = sysconf(_SC_PAGESIZE);
    if (page <= 0) return fail(JF_STATUS_IO_ERROR, "query system page size: %s", strerror(errno));
    uint64_t * sums = calloc(model->file_count > 0 ? model->file_count : 1, sizeof(*sums));
    if (sums == NULL) return fail(JF_STATUS_OUT_OF_MEMORY, "allocate prefetch checksums");
    prefetch_job job;
    job.model = model;
    job.page = (size_t) page;
    atomic_init(&job.next_file, 0);
    job.file_sums = sums;
    const size_t workers = model->file_count < thread_count ? model->file_count : thread_count;
    pthread_t threads[256];
    size_t started = 0;
    for (; started + 1 < workers; ++started) {
        if (pthread_create(&threads[started], NULL, prefetch_worker, &job) != 0) break;
    }
    (void) prefetch_worker(&job);
    for (size_t i = 0; i < started; ++i) pthread_join(threads[i], NULL);
    if (workers > 0 && started + 1 < workers) {
        free(sums);
        return fail(JF_STATUS_IO_ERROR, "create prefetch worker thread");
    }
    uint64_t h = 0xcbf29ce484222325ull;
    for (size_t f = 0; f < model->file_count; ++f) h = (h ^ sums[f]) * 0x100000001b3ull;
    free(sums);
    if (checksum != NULL) *checksum = h;
    return ok_status();
}

jf_status jf_model_prefetch(jf_model * model, uint64_t * checksum) {
    return jf_model_prefetch_parallel(model, 1, checksum);
}

const char * jf_status_code_name(jf_status_code code) {
    switch (code) {
    case JF_STATUS_OK: return "ok";
    case JF_STATUS_INVALID_ARGUMENT: return "invalid_argument";
    case JF_STATUS_IO_ERROR: return "io_error";
    case JF_STATUS_FORMAT_ERROR: return "format_error";
    case JF_STATUS_NOT_FOUND: return "not_found";
    case JF_STATUS_OUT_OF_MEMORY: return "out_of_memory";
    }
    return "unknown";
}
