// SPDX-License-Identifier: Unlicense
//
// Weight-file reader (pth_loader.h): safetensors (8-byte little-endian
// header length, JSON header of {name: {dtype, shape, data_offsets}},
// then the data), with the reference's pth_* entry points and their
// fatal-on-error behaviour (pth_loader.c:1148-1403 of the reference, whose
// torch.save zip reader is not part of this build).

#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

#include "common.cuh"
#include "pth_loader.h"

using coreg::fail;
using coreg::pending;

namespace {

// Minimal JSON reader for the safetensors header: objects, arrays,
// strings, numbers (and the literals true / false / null, skipped).
struct Json {
    const char *s, *e;
    bool bad = false;

    void ws()
    {
        while (s < e && (*s == ' ' || *s == '\n' || *s == '\r' || *s == '\t'))
            s++;
    }
    bool eat(char c)
    {
        ws();
        if (s < e && *s == c) {
            s++;
            return true;
        }
        return false;
    }
    bool str(std::string &out)
    {
        ws();
        if (s >= e || *s != '"')
            return bad = true, false;
        s++;
        out.clear();
        while (s < e && *s != '"') {
            if (*s == '\\' && s + 1 < e) {
                s++;
                char c = *s;
                out += c == 'n' ? '\n' : c == 't' ? '\t' : c;
            }
            else
                out += *s;
            s++;
        }
        if (s >= e)
            return bad = true, false;
        s++;
        return true;
    }
    bool num(long &v)
    {
        ws();
        char *end;
        v = strtol(s, &end, 10);
        if (end == s)
            return bad = true, false;
        s = end;
        return true;
    }
    void skip()
    {
        ws();
        if (s >= e) {
            bad = true;
            return;
        }
        if (*s == '"') {
            std::string t;
            str(t);
        }
        else if (*s == '{' || *s == '[') {
            const char close = *s == '{' ? '}' : ']';
            s++;
            if (eat(close))
                return;
            do {
                if (close == '}') {
                    std::string k;
                    str(k);
                    if (!eat(':')) {
                        bad = true;
                        return;
                    }
                }
                skip();
            } while (!bad && eat(','));
            if (!eat(close))
                bad = true;
        }
        else
            while (s < e && *s != ',' && *s != '}' && *s != ']')
                s++;
    }
};

}  // namespace

extern "C" void pth_open(struct pth_file *pf, const char *path)
{
    unsigned char hdr8[8];
    uint64_t hlen = 0;
    std::vector<char> buf;
    std::vector<struct pth_tensor> ts;
    Json j;

    memset(pf, 0, sizeof(*pf));
    if (pending())
        return;
    FILE *fp = fopen(path, "rb");
    if (!fp) {
        fail("Unable to open checkpoint <%s>", path);
        return;
    }
    if (fread(hdr8, 1, 8, fp) != 8) {
        fclose(fp);
        fail("Checkpoint <%s> is too short", path);
        return;
    }
    if (hdr8[0] == 'P' && hdr8[1] == 'K') {
        fclose(fp);
        fail("Checkpoint <%s> is a torch.save zip archive; this build reads "
             "safetensors files",
             path);
        return;
    }
    for (int i = 7; i >= 0; i--)
        hlen = hlen << 8 | hdr8[i];
    if (hlen == 0 || hlen > ((uint64_t)1 << 30)) {
        fclose(fp);
        fail("Checkpoint <%s>: not a safetensors file", path);
        return;
    }
    buf.resize(hlen);
    if (fread(buf.data(), 1, hlen, fp) != hlen) {
        fclose(fp);
        fail("Checkpoint <%s>: truncated header", path);
        return;
    }
    j.s = buf.data();
    j.e = buf.data() + hlen;
    if (!j.eat('{')) {
        fclose(fp);
        fail("Checkpoint <%s>: header is not a JSON object", path);
        return;
    }
    const off_t base = 8 + (off_t)hlen;
    if (!j.eat('}'))
        do {
            std::string name;
            if (!j.str(name) || !j.eat(':'))
                break;
            if (name == "__metadata__") {
                j.skip();
                continue;
            }
            struct pth_tensor t;
            memset(&t, 0, sizeof(t));
            long off0 = -1, off1 = -1;
            std::string dtype;
            if (!j.eat('{')) {
                j.bad = true;
                break;
            }
            do {
                std::string key;
                if (!j.str(key) || !j.eat(':'))
                    break;
                if (key == "dtype")
                    j.str(dtype);
                else if (key == "shape") {
                    if (!j.eat('['))
                        j.bad = true;
                    else if (!j.eat(']')) {
                        do {
                            long v;
                            if (!j.num(v))
                                break;
                            if (t.ndim >= PTH_MAX_DIMS) {
                                j.bad = true;
                                break;
                            }
                            t.shape[t.ndim++] = v;
                        } while (j.eat(','));
                        if (!j.eat(']'))
                            j.bad = true;
                    }
                }
                else if (key == "data_offsets") {
                    if (!j.eat('[') || !j.num(off0) || !j.eat(',') ||
                        !j.num(off1) || !j.eat(']'))
                        j.bad = true;
                }
                else
                    j.skip();
            } while (!j.bad && j.eat(','));
            if (j.bad || !j.eat('}'))
                break;
            t.dtype = dtype == "F32"    ? PTH_F32
                      : dtype == "F16"  ? PTH_F16
                      : dtype == "BF16" ? PTH_BF16
                                        : PTH_OTHER;
            if (off0 < 0 || off1 < off0) {
                j.bad = true;
                break;
            }
            long st = 1;
            for (int d = t.ndim - 1; d >= 0; d--) {
                t.stride[d] = st;
                st *= t.shape[d];
            }
            t.data_offset = base + off0;
            t.storage_bytes = (size_t)(off1 - off0);
            t.name = strdup(name.c_str());
            ts.push_back(t);
        } while (!j.bad && j.eat(','));
    if (j.bad) {
        for (auto &t : ts)
            free(t.name);
        fclose(fp);
        fail("Checkpoint <%s>: malformed safetensors header", path);
        return;
    }
    pf->fp = fp;
    pf->path = strdup(path);
    pf->ntensors = (int)ts.size();
    pf->tensors = (struct pth_tensor *)malloc(ts.size() * sizeof(ts[0]) + 1);
    memcpy(pf->tensors, ts.data(), ts.size() * sizeof(ts[0]));
}

extern "C" const struct pth_tensor *pth_find(const struct pth_file *pf,
                                             const char *name)
{
    for (int i = 0; i < pf->ntensors; i++)
        if (!strcmp(pf->tensors[i].name, name))
            return &pf->tensors[i];
    return NULL;
}

extern "C" int pth_strip_prefix(struct pth_file *pf, const char *prefix)
{
    const size_t n = strlen(prefix);
    int k = 0;
    for (int i = 0; i < pf->ntensors; i++) {
        char *name = pf->tensors[i].name;
        if (!strncmp(name, prefix, n)) {
            memmove(name, name + n, strlen(name + n) + 1);
            k++;
        }
    }
    return k;
}

extern "C" const struct pth_tensor *pth_require(const struct pth_file *pf,
                                                const char *name, int ndim,
                                                const long *shape)
{
    const struct pth_tensor *t = pth_find(pf, name);
    if (pending())
        return NULL;
    if (!t) {
        fail("Tensor <%s> not found in checkpoint <%s>", name, pf->path);
        return NULL;
    }
    if (t->ndim != ndim) {
        fail("Tensor <%s> has rank %d, expected %d", name, t->ndim, ndim);
        return NULL;
    }
    for (int d = 0; d < ndim; d++)
        if (shape && shape[d] >= 0 && t->shape[d] != shape[d]) {
            fail("Tensor <%s> has size %ld along axis %d, expected %ld", name,
                 t->shape[d], d, shape[d]);
            return NULL;
        }
    return t;
}

extern "C" long pth_numel(const struct pth_tensor *t)
{
    long n = 1;
    for (int d = 0; d < t->ndim; d++)
        n *= t->shape[d];
    return n;
}

extern "C" double pth_bytes(const struct pth_file *pf, const char *prefix)
{
    const size_t n = strlen(prefix);
    double s = 0;
    for (int i = 0; i < pf->ntensors; i++)
        if (!strncmp(pf->tensors[i].name, prefix, n))
            s += (double)pf->tensors[i].storage_bytes;
    return s;
}

static float half_bits(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0)
            u = sign;
        else {
            // Subnormal: normalize.
            int sh = 0;
            while (!(m & 0x400)) {
                m <<= 1;
                sh++;
            }
            m &= 0x3ff;
            u = sign | (uint32_t)(127 - 15 - sh + 1) << 23 | m << 13;
        }
    }
    else if (e == 31)
        u = sign | 0x7f800000u | m << 13;
    else
        u = sign | (e + 127 - 15) << 23 | m << 13;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

extern "C" float *pth_read_f32(const struct pth_file *pf,
                               const struct pth_tensor *t)
{
    if (pending() || !t)
        return NULL;
    const long n = pth_numel(t);
    const int es = t->dtype == PTH_F32 ? 4 : 2;
    if (t->dtype == PTH_OTHER) {
        fail("Tensor <%s>: not a floating-point tensor", t->name);
        return NULL;
    }
    if ((size_t)n * es > t->storage_bytes) {
        fail("Tensor <%s>: %ld elements do not fit its %zu bytes", t->name, n,
             t->storage_bytes);
        return NULL;
    }
    float *out = (float *)malloc((size_t)(n > 0 ? n : 1) * sizeof(float));
    if (fseeko(pf->fp, t->data_offset, SEEK_SET) != 0) {
        free(out);
        fail("Tensor <%s>: seek failed in <%s>", t->name, pf->path);
        return NULL;
    }
    if (t->dtype == PTH_F32) {
        if (fread(out, 4, (size_t)n, pf->fp) != (size_t)n) {
            free(out);
            fail("Tensor <%s>: read failed in <%s>", t->name, pf->path);
            return NULL;
        }
        return out;
    }
    std::vector<uint16_t> h((size_t)n);
    if (fread(h.data(), 2, (size_t)n, pf->fp) != (size_t)n) {
        free(out);
        fail("Tensor <%s>: read failed in <%s>", t->name, pf->path);
        return NULL;
    }
    for (long i = 0; i < n; i++) {
        if (t->dtype == PTH_F16)
            out[i] = half_bits(h[i]);
        else {
            const uint32_t u = (uint32_t)h[i] << 16;
            memcpy(&out[i], &u, 4);
        }
    }
    return out;
}

extern "C" void pth_close(struct pth_file *pf)
{
    if (pf->fp)
        fclose(pf->fp);
    for (int i = 0; i < pf->ntensors; i++)
        free(pf->tensors[i].name);
    free(pf->tensors);
    free(pf->path);
    memset(pf, 0, sizeof(*pf));
}
