// Test infrastructure: a C shim over the reference's own GGUF reader (stbl/gguf.h, stbl/gguf.cpp,
// compiled from the reference tree by build_ref.sh into _ref/libstbl_ref_gguf.so), so the tests can
// compare the library's reader (include/stbl_gguf.h) with it on the same files.  Not part of the
// product; nothing outside tests/ loads it.
#include <string.h>

#include <string>

#include "gguf.h"

extern "C" {

void *ref_gguf_open(const char *path, char *err, int errlen) {
    GgufFile *f = new GgufFile();
    std::string e;
    if (!f->open(path, e)) {
        strncpy(err, e.c_str(), (size_t)errlen - 1);
        err[errlen - 1] = 0;
        delete f;
        return nullptr;
    }
    return f;
}

void ref_gguf_close(void *h) { delete static_cast<GgufFile *>(h); }

int ref_gguf_n_tensors(void *h) { return (int)static_cast<GgufFile *>(h)->tensors.size(); }

// tensor i in the reader's own (name) order
int ref_gguf_tensor_at(void *h, int i, char *name, int namecap, uint32_t *type, uint32_t *n_dims, uint64_t *dims,
                       uint64_t *offset, uint64_t *nbytes) {
    GgufFile *f = static_cast<GgufFile *>(h);
    auto it = f->tensors.begin();
    for (int k = 0; k < i && it != f->tensors.end(); k++) ++it;
    if (it == f->tensors.end()) return -1;
    const GgufTensor &t = it->second;
    strncpy(name, t.name.c_str(), (size_t)namecap - 1);
    name[namecap - 1] = 0;
    *type = t.type;
    *n_dims = (uint32_t)t.dims.size();
    for (size_t d = 0; d < 4; d++) dims[d] = d < t.dims.size() ? t.dims[d] : 1;
    *offset = t.offset;
    *nbytes = t.nbytes;
    return 0;
}

int ref_gguf_u32(void *h, const char *key, uint32_t *v) {
    try {
        *v = static_cast<GgufFile *>(h)->u32(key);
        return 0;
    } catch (...) {
        return -1;
    }
}

int ref_gguf_f32(void *h, const char *key, float *v) {
    try {
        *v = static_cast<GgufFile *>(h)->f32(key);
        return 0;
    } catch (...) {
        return -1;
    }
}

}  // extern "C"
