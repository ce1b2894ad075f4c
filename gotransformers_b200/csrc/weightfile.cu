// weightfile.cu -- GoTransformers binary weights files straight into a handle.
//
// A saved model (weightfile.SaveBinaryWithPrecision, weightfile/binaryfile.go:
// 27-52) is a marker, a parameter count and one record per parameter: a name
// and its values -- float64 in version 1 (:75-82); in version 2 (:84-95) a
// storage byte, then float64 / float32 / bfloat16 values or a compressed-rows
// record (:127-138: precision, rows, width and the five count-prefixed lists
// of lowprecision.RowsSnapshot).  gtmoe_weightfile_open maps the file and
// indexes the records the way ReadBinaryKeepingCompressed walks them
// (:157-230), with the same checks (:232-398, lowprecision/rows.go:172-203);
// the setters hand the mapped RowsSnapshot bytes to gtmoe_set_expert_layer /
// gtmoe_set_router, which copy them to the device: the compressed rows never
// pass through a decoded host copy.  Host code only.
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "handle.h"

namespace gtmoe {
namespace {

const char kMarkerV1[] = "GOTRANSFORMERS-WEIGHTS-1";
const char kMarkerV2[] = "GOTRANSFORMERS-WEIGHTS-2";
constexpr size_t kMarkerLen = sizeof(kMarkerV1) - 1;

enum StoredAs { kFloat64 = 1, kFloat32 = 2, kBFloat16 = 3, kCompressedRows = 4 };

// One count-prefixed list inside the mapping.
struct List {
    const uint8_t *p = nullptr;
    uint64_t count = 0;
};

struct Param {
    std::string name;
    int stored_as = kFloat64;
    List values;  // dense parameters
    // compressed rows
    int precision = 0;
    uint64_t rows = 0, width = 0;
    List f64, f32, i8, fp4, scales;
};

uint64_t scale_blocks_of(uint64_t width) { return (width + 15) / 16; }

}  // namespace
}  // namespace gtmoe

struct gtmoe_weightfile {
    std::string path;
    int fd = -1;
    const uint8_t *base = nullptr;
    uint64_t size = 0;
    std::vector<gtmoe::Param> params;
    std::unordered_map<std::string, size_t> by_name;
};

namespace gtmoe {
using WeightFile = gtmoe_weightfile;
namespace {

// Sequential reader over the mapping; every read is bounds-checked (the Go
// reader gets an io error where this one runs past the end).
struct Reader {
    const WeightFile &wf;
    uint64_t off = 0;
    bool take(uint64_t n, const uint8_t **p) {
        if (n > wf.size - off) return false;
        *p = wf.base + off;
        off += n;
        return true;
    }
    template <typename T>
    bool scalar(T *v) {
        const uint8_t *p;
        if (!take(sizeof(T), &p)) return false;
        memcpy(v, p, sizeof(T));
        return true;
    }
};

// readCount + readList (binaryfile.go:247-270): a uint64 count no larger than
// the file could hold, then the values.
int read_list(Reader &r, const std::string &name, const char *what, uint64_t bytes_per_value, List *out) {
    const WeightFile &wf = r.wf;
    uint64_t count = 0;
    if (!r.scalar(&count))
        return fail(GTMOE_EINVAL, "%s: could not read the %s count of parameter \"%s\"", wf.path.c_str(), what,
                    name.c_str());
    if (count > wf.size / bytes_per_value)
        return fail(GTMOE_EINVAL, "%s: parameter \"%s\" says it has %llu %s, which is more than the file can hold",
                    wf.path.c_str(), name.c_str(), (unsigned long long)count, what);
    const uint8_t *p = nullptr;
    if (count > 0 && !r.take(count * bytes_per_value, &p))
        return fail(GTMOE_EINVAL, "%s: could not read the %s of parameter \"%s\"", wf.path.c_str(), what,
                    name.c_str());
    out->p = p;
    out->count = count;
    return 0;
}

int parse(WeightFile &wf) {
    Reader r{wf};
    const uint8_t *marker;
    if (!r.take(kMarkerLen, &marker)) return fail(GTMOE_EINVAL, "%s: this is not a binary weights file", wf.path.c_str());
    const bool v1 = memcmp(marker, kMarkerV1, kMarkerLen) == 0;
    if (!v1 && memcmp(marker, kMarkerV2, kMarkerLen) != 0)
        return fail(GTMOE_EINVAL, "%s: this is not a binary weights file", wf.path.c_str());
    uint32_t n = 0;
    if (!r.scalar(&n))
        return fail(GTMOE_EINVAL, "%s: could not read how many parameters are saved", wf.path.c_str());
    for (uint32_t i = 0; i < n; i++) {
        Param p;
        uint32_t len = 0;
        if (!r.scalar(&len))
            return fail(GTMOE_EINVAL, "%s: could not read the name length of parameter %u", wf.path.c_str(), i);
        if ((uint64_t)len > wf.size)
            return fail(GTMOE_EINVAL, "%s: parameter %u says its name is %u bytes long, which is bigger than the file",
                        wf.path.c_str(), i, len);
        const uint8_t *nm;
        if (!r.take(len, &nm))
            return fail(GTMOE_EINVAL, "%s: could not read the name of parameter %u", wf.path.c_str(), i);
        p.name.assign((const char *)nm, len);
        if (wf.by_name.count(p.name))
            return fail(GTMOE_EINVAL, "%s: parameter \"%s\" is in the file twice", wf.path.c_str(), p.name.c_str());
        if (v1) {
            p.stored_as = kFloat64;
            GT_CHECK(read_list(r, p.name, "values", 8, &p.values));
        } else {
            uint8_t stored = 0;
            if (!r.scalar(&stored))
                return fail(GTMOE_EINVAL, "%s: could not read how parameter \"%s\" is stored", wf.path.c_str(),
                            p.name.c_str());
            p.stored_as = stored;
            switch (stored) {
                case kFloat64: GT_CHECK(read_list(r, p.name, "values", 8, &p.values)); break;
                case kFloat32: GT_CHECK(read_list(r, p.name, "float32 values", 4, &p.values)); break;
                case kBFloat16: GT_CHECK(read_list(r, p.name, "bfloat16 values", 2, &p.values)); break;
                case kCompressedRows: {
                    // readCompressedRows (binaryfile.go:356-398)
                    uint8_t prec = 0;
                    if (!r.scalar(&prec))
                        return fail(GTMOE_EINVAL, "%s: could not read the precision of compressed parameter \"%s\"",
                                    wf.path.c_str(), p.name.c_str());
                    if (!r.scalar(&p.rows))
                        return fail(GTMOE_EINVAL, "%s: could not read the row count of compressed parameter \"%s\"",
                                    wf.path.c_str(), p.name.c_str());
                    if (!r.scalar(&p.width))
                        return fail(GTMOE_EINVAL, "%s: could not read the row width of compressed parameter \"%s\"",
                                    wf.path.c_str(), p.name.c_str());
                    const uint64_t most = 2 * wf.size;
                    if (p.width == 0 || p.width > most || p.rows > most / p.width)
                        return fail(GTMOE_EINVAL,
                                    "%s: compressed parameter \"%s\" says it is %llu rows of %llu values, which does "
                                    "not fit in the file",
                                    wf.path.c_str(), p.name.c_str(), (unsigned long long)p.rows,
                                    (unsigned long long)p.width);
                    p.precision = prec;
                    GT_CHECK(read_list(r, p.name, "float64 values", 8, &p.f64));
                    GT_CHECK(read_list(r, p.name, "float32 values", 4, &p.f32));
                    GT_CHECK(read_list(r, p.name, "int8 values", 1, &p.i8));
                    GT_CHECK(read_list(r, p.name, "fp4 values", 1, &p.fp4));
                    GT_CHECK(read_list(r, p.name, "scales", 4, &p.scales));
                    // RowsFromSnapshot (lowprecision/rows.go:172-203)
                    if (prec > GTMOE_FP4)
                        return fail(GTMOE_EINVAL, "%s: compressed parameter \"%s\": rows snapshot has an unknown precision %d",
                                    wf.path.c_str(), p.name.c_str(), prec);
                    const uint64_t blocks = scale_blocks_of(p.width);
                    uint64_t have = 0, want = 0;
                    switch (prec) {
                        case GTMOE_FLOAT64: have = p.f64.count * 8, want = p.rows * p.width * 8; break;
                        case GTMOE_FLOAT32: have = p.f32.count * 4, want = p.rows * p.width * 4; break;
                        case GTMOE_INT8:
                            have = p.i8.count + p.scales.count * 4, want = p.rows * (p.width + blocks * 4);
                            break;
                        default:
                            have = p.fp4.count + p.scales.count * 4, want = p.rows * ((p.width + 1) / 2 + blocks * 4);
                    }
                    if (have != want)
                        return fail(GTMOE_EINVAL,
                                    "%s: compressed parameter \"%s\": rows snapshot for %llu rows of width %llu has the "
                                    "wrong amount of data",
                                    wf.path.c_str(), p.name.c_str(), (unsigned long long)p.rows,
                                    (unsigned long long)p.width);
                    // RowsFromSnapshot checks only that combined count, so a
                    // snapshot with, say, fewer scales and more codes passes it
                    // and the reference panics later, when DotRow indexes past
                    // the shorter list.  Such a record is damaged either way;
                    // it is refused here, before any layer setter could read
                    // past the end of a list.
                    {
                        uint64_t codes = 0, want_codes = p.rows * p.width, want_scales = 0;
                        switch (prec) {
                            case GTMOE_FLOAT64: codes = p.f64.count; break;
                            case GTMOE_FLOAT32: codes = p.f32.count; break;
                            case GTMOE_INT8: codes = p.i8.count, want_scales = p.rows * blocks; break;
                            default:
                                codes = p.fp4.count, want_codes = p.rows * ((p.width + 1) / 2),
                                want_scales = p.rows * blocks;
                        }
                        if (codes != want_codes || p.scales.count != want_scales)
                            return fail(GTMOE_EINVAL,
                                        "%s: compressed parameter \"%s\": rows snapshot holds %llu codes and %llu "
                                        "scales; %llu rows of width %llu need %llu and %llu",
                                        wf.path.c_str(), p.name.c_str(), (unsigned long long)codes,
                                        (unsigned long long)p.scales.count, (unsigned long long)p.rows,
                                        (unsigned long long)p.width, (unsigned long long)want_codes,
                                        (unsigned long long)want_scales);
                    }
                    break;
                }
                default:
                    return fail(GTMOE_EINVAL, "%s: parameter \"%s\" is stored in an unknown way (%d)",
                                wf.path.c_str(), p.name.c_str(), stored);
            }
        }
        wf.by_name[p.name] = wf.params.size();
        wf.params.push_back(std::move(p));
    }
    return 0;
}

// A dense parameter's values as float64 (readFloat32Values / readBFloat16Values,
// binaryfile.go:318-340: float32 widened, bfloat16 bits << 16 as a float32).
std::vector<double> dense_values(const Param &p) {
    std::vector<double> v(p.values.count);
    for (uint64_t i = 0; i < p.values.count; i++) {
        if (p.stored_as == kFloat64) {
            memcpy(&v[i], p.values.p + 8 * i, 8);
        } else if (p.stored_as == kFloat32) {
            float f;
            memcpy(&f, p.values.p + 4 * i, 4);
            v[i] = f;
        } else {
            uint16_t b;
            memcpy(&b, p.values.p + 2 * i, 2);
            uint32_t u = (uint32_t)b << 16;
            float f;
            memcpy(&f, &u, 4);
            v[i] = f;
        }
    }
    return v;
}

int find(const WeightFile *wf, const char *name, const Param **out) {
    if (!name) return fail(GTMOE_EINVAL, "parameter name is NULL");
    auto it = wf->by_name.find(name);
    if (it == wf->by_name.end())
        return fail(GTMOE_EINVAL, "%s: there is no parameter \"%s\"", wf->path.c_str(), name);
    *out = &wf->params[it->second];
    return 0;
}

// The RowsSnapshot lists of a compressed parameter, or a dense parameter of
// rows x width values (widened to float64), as the setters take them.
struct LayerSource {
    int precision = GTMOE_FLOAT64;
    const void *values = nullptr;
    const float *scales = nullptr;
    std::vector<double> dense;   // dense parameters and unaligned float64 rows
    std::vector<float> aligned;  // unaligned float32 lists
    std::vector<float> scales_aligned;
};

template <typename T>
const T *aligned_copy(const List &l, std::vector<T> &buf) {
    if ((reinterpret_cast<uintptr_t>(l.p) % alignof(T)) == 0) return reinterpret_cast<const T *>(l.p);
    buf.resize(l.count);
    memcpy(buf.data(), l.p, l.count * sizeof(T));
    return buf.data();
}

int layer_source(const WeightFile *wf, const Param &p, uint64_t rows, uint64_t width, LayerSource *s) {
    if (p.stored_as != kCompressedRows) {
        if (p.values.count != rows * width)
            return fail(GTMOE_EINVAL, "%s: parameter \"%s\" has %llu values, the layer needs %llu x %llu",
                        wf->path.c_str(), p.name.c_str(), (unsigned long long)p.values.count,
                        (unsigned long long)rows, (unsigned long long)width);
        s->precision = GTMOE_FLOAT64;
        s->dense = dense_values(p);
        s->values = s->dense.data();
        return 0;
    }
    if (p.rows != rows || p.width != width)
        return fail(GTMOE_EINVAL, "%s: parameter \"%s\" is %llu x %llu, the layer needs %llu x %llu", wf->path.c_str(),
                    p.name.c_str(), (unsigned long long)p.rows, (unsigned long long)p.width,
                    (unsigned long long)rows, (unsigned long long)width);
    s->precision = p.precision;
    switch (p.precision) {
        case GTMOE_FLOAT64: s->values = aligned_copy<double>(p.f64, s->dense); break;
        case GTMOE_FLOAT32: s->values = aligned_copy<float>(p.f32, s->aligned); break;
        case GTMOE_INT8: s->values = p.i8.p; break;
        default: s->values = p.fp4.p;
    }
    if (p.precision == GTMOE_INT8 || p.precision == GTMOE_FP4) s->scales = aligned_copy<float>(p.scales, s->scales_aligned);
    return 0;
}

int bias_values(const WeightFile *wf, const char *name, uint64_t n, std::vector<double> *out) {
    if (!name) return 0;
    const Param *p;
    GT_CHECK(find(wf, name, &p));
    if (p->stored_as == kCompressedRows)
        return fail(GTMOE_EINVAL, "%s: bias \"%s\" is stored as compressed rows", wf->path.c_str(), name);
    if (p->values.count != n)
        return fail(GTMOE_EINVAL, "%s: bias \"%s\" has %llu values, the layer has %llu outputs", wf->path.c_str(), name,
                    (unsigned long long)p->values.count, (unsigned long long)n);
    *out = dense_values(*p);
    return 0;
}

}  // namespace
}  // namespace gtmoe

using namespace gtmoe;

extern "C" {

int gtmoe_weightfile_open(const char *path, gtmoe_wf_t *out) {
    if (!path || !out) return fail(GTMOE_EINVAL, "path or out is NULL");
    *out = nullptr;
    WeightFile *wf = new WeightFile();
    wf->path = path;
    wf->fd = open(path, O_RDONLY);
    if (wf->fd < 0) {
        delete wf;
        return fail(GTMOE_EINVAL, "%s: could not open the file", path);
    }
    struct stat sb;
    if (fstat(wf->fd, &sb) != 0) {
        close(wf->fd);
        delete wf;
        return fail(GTMOE_EINVAL, "%s: could not read the file size", path);
    }
    wf->size = (uint64_t)sb.st_size;
    if (wf->size > 0) {
        void *m = mmap(nullptr, wf->size, PROT_READ, MAP_PRIVATE, wf->fd, 0);
        if (m == MAP_FAILED) {
            close(wf->fd);
            delete wf;
            return fail(GTMOE_EINVAL, "%s: could not map the file", path);
        }
        wf->base = (const uint8_t *)m;
    }
    int rc = parse(*wf);
    if (rc != 0) {
        gtmoe_weightfile_close(wf);
        return rc;
    }
    *out = wf;
    return 0;
}

void gtmoe_weightfile_close(gtmoe_wf_t wf) {
    if (!wf) return;
    if (wf->base) munmap((void *)wf->base, wf->size);
    if (wf->fd >= 0) close(wf->fd);
    delete wf;
}

int gtmoe_weightfile_count(gtmoe_wf_t wf) { return wf ? (int)wf->params.size() : 0; }

int gtmoe_weightfile_info(gtmoe_wf_t wf, int i, const char **name, int *stored_as, int *precision, int64_t *rows,
                          int64_t *width, int64_t *values) {
    if (!wf) return fail(GTMOE_EINVAL, "weight file is NULL");
    if (i < 0 || i >= (int)wf->params.size()) return fail(GTMOE_EINVAL, "parameter %d out of range", i);
    const Param &p = wf->params[i];
    if (name) *name = p.name.c_str();
    if (stored_as) *stored_as = p.stored_as;
    const bool rows_rec = p.stored_as == kCompressedRows;
    if (precision) *precision = rows_rec ? p.precision : -1;
    if (rows) *rows = rows_rec ? (int64_t)p.rows : 0;
    if (width) *width = rows_rec ? (int64_t)p.width : 0;
    if (values) *values = rows_rec ? (int64_t)(p.rows * p.width) : (int64_t)p.values.count;
    return 0;
}

int gtmoe_weightfile_set_expert_layer(gtmoe_wf_t wf, gtmoe_t h, int kind, int index, int which, const char *weights,
                                      const char *bias) {
    if (!wf || !h) return fail(GTMOE_EINVAL, "weight file or handle is NULL");
    if (which < GTMOE_GATE || which > GTMOE_DOWN) return fail(GTMOE_EINVAL, "unknown layer %d", which);
    const uint64_t d = h->cfg.d_model, hd = h->cfg.hidden;
    const uint64_t rows = which == GTMOE_DOWN ? d : hd, width = which == GTMOE_DOWN ? hd : d;
    const Param *p;
    GT_CHECK(find(wf, weights, &p));
    LayerSource src;
    GT_CHECK(layer_source(wf, *p, rows, width, &src));
    std::vector<double> b;
    GT_CHECK(bias_values(wf, bias, rows, &b));
    return gtmoe_set_expert_layer(h, kind, index, which, src.precision, src.values, src.scales, (int)rows, (int)width,
                                  bias ? b.data() : nullptr);
}

int gtmoe_weightfile_set_router(gtmoe_wf_t wf, gtmoe_t h, const char *weights, const char *bias) {
    if (!wf || !h) return fail(GTMOE_EINVAL, "weight file or handle is NULL");
    const uint64_t E = h->cfg.n_routed, d = h->cfg.d_model;
    const Param *p;
    GT_CHECK(find(wf, weights, &p));
    LayerSource src;
    GT_CHECK(layer_source(wf, *p, E, d, &src));
    std::vector<double> b;
    GT_CHECK(bias_values(wf, bias, E, &b));
    return gtmoe_set_router(h, src.precision, src.values, src.scales, bias ? b.data() : nullptr);
}

}  // extern "C"
