/* GGUF container reader: the reference engine's checkpoint format, the data format on the input side
 * of the MoE layer path.
 *
 * Replaces the reference's GgufFile (stbl/gguf.h:17-31, stbl/gguf.cpp:58-148): the file is mapped read
 * only, the metadata table and the tensor table are parsed once, and tensors are handed out as
 * pointers into the mapping.  The layer loader (stblarge_b200/gguf.py: load_moe_layer) takes a layer's
 * router (blk.N.ffn_gate_inp.weight, exp_probs_b.bias), FP8-e8m0 shared expert
 * (blk.N.ffn_{gate,up,down}_shexp.{weight,scale}) and MXFP4 routed experts
 * (blk.N.ffn_{gate,up,down}_exps.weight, 17-byte blocks) from here, as the reference's model loader
 * does (stbl/model.cu:933-947), and converts the expert blocks on the device (stbl_mxfp4_from_gguf).
 *
 * Accepted: GGUF versions 2 and 3 (64-bit counts), every metadata value type (0-12, nested arrays
 * included), tensors of at most 4 dimensions of the types F32 (0), F16 (1), Q8_0 (8), I8 (24), BF16
 * (30), MXFP4 (39), and the reference's STBL_E4M3 (200) and STBL_E8M0 (201).  Rejected with an error
 * (where the reference reads on): a version other than 2 or 3, a tensor type or dimension count it
 * cannot size, an element count not a multiple of the type's block, a duplicated tensor name, an
 * alignment that is 0 or not a u32, a tensor whose data ends past the file.  Plain C types only; no
 * function throws; the handle is not thread-safe for close. */
#ifndef STBL_GGUF_H
#define STBL_GGUF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct stbl_gguf stbl_gguf;

/* GGUF tensor type ids this reader sizes (ggml ids, plus the reference's FP8 pair). */
enum {
    STBL_GGUF_F32 = 0,
    STBL_GGUF_F16 = 1,
    STBL_GGUF_Q8_0 = 8,
    STBL_GGUF_I8 = 24,
    STBL_GGUF_BF16 = 30,
    STBL_GGUF_MXFP4 = 39,
    STBL_GGUF_STBL_E4M3 = 200,
    STBL_GGUF_STBL_E8M0 = 201,
};

typedef struct {
    const char *name;  /* valid while the file is open */
    uint32_t type;
    uint32_t n_dims;
    uint64_t dims[4];  /* GGUF order: dims[0] is the contiguous (innermost) dimension; unused dims 1 */
    uint64_t offset;   /* absolute file offset of the data */
    uint64_t nbytes;
    const void *data;  /* inside the read-only mapping */
} stbl_gguf_tensor;

/* Maps and parses `path`.  0 and *out on success; -1 and a message in err otherwise. */
int stbl_gguf_open(const char *path, stbl_gguf **out, char *err, int errlen);
void stbl_gguf_close(stbl_gguf *g);

/* File version, the data alignment and the number of metadata records and tensors. */
int stbl_gguf_info(const stbl_gguf *g, uint32_t *version, uint64_t *alignment, uint64_t *n_kv, uint64_t *n_tensors);

/* Tensor i in file order / by name (the reference's GgufFile::tensor).  0, or -1 when absent. */
int stbl_gguf_tensor_at(const stbl_gguf *g, uint64_t i, stbl_gguf_tensor *t);
int stbl_gguf_find(const stbl_gguf *g, const char *name, stbl_gguf_tensor *t);

/* Metadata record i: its key (valid while open) and value type (0-12). */
int stbl_gguf_kv_at(const stbl_gguf *g, uint64_t i, const char **key, uint32_t *type);

/* Typed metadata values (GgufFile::u32 / f32 / uints): 0, or -1 when the key is missing or of another
 * type.  stbl_gguf_uints takes a u32 or u64 array, writes min(n, cap) values and returns n (-1 on error).
 * stbl_gguf_str copies at most cap - 1 bytes and a terminating 0, and returns the string's length. */
int stbl_gguf_u32(const stbl_gguf *g, const char *key, uint32_t *v);
int stbl_gguf_f32(const stbl_gguf *g, const char *key, float *v);
int64_t stbl_gguf_uints(const stbl_gguf *g, const char *key, uint64_t *v, int64_t cap);
int64_t stbl_gguf_str(const stbl_gguf *g, const char *key, char *buf, int64_t cap);

#ifdef __cplusplus
}
#endif

#endif
