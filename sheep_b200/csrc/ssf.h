// SSF ("Sheep Standard Format") on-disk structures and the engine's loader.
//
// The byte layout below is fixed by the format, so the two packed structs
// follow the reference definitions field for field (sml/sml-model.h:83-203,
// tooling/sml_format.py:53-96 HEADER_FMT / REC_FMT). Everything else here --
// the loader, the validation order, the view types -- is this engine's own.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SSF_NAME_LEN      64
#define SSF_MAX_LEVELS    4
#define SSF_HEADER_BYTES  4096u
#define SSF_MAX_VERSION   9
#define SSF_GROUP         32      // weights per group (one scale and min field)
#define SSF_SUPER         256     // weights per superblock (one fp16 d and md)
#define SSF_GPS           8       // groups per superblock

#define SSF_KIND_F32      0u
#define SSF_KIND_QUANT    1u      // "LADDER" kind in the reference: any coded tensor
#define SSF_LAYOUT_LADDER 0u
#define SSF_LAYOUT_FLAT   1u

#define SSF_FLAG_HADAMARD 1u
#define SSF_FLAG_SCALE6   2u      // v9: 6-bit group fields, 4 groups per 3 bytes
#define SSF_FLAG_MINNEG   4u      // with SCALE6: min field read as (f - 63) * md
#define SSF_FLAG_EXACT    8u

#pragma pack(push, 1)
typedef struct {
    char     name[SSF_NAME_LEN];
    uint32_t kind, rows, cols, group;
    uint64_t off, nbytes;          // f32 payload
    uint64_t sd_off, sd_n;         // fp16 step scale per superblock
    uint64_t sq_off, sq_n;         // step field per group
    uint64_t perm_off, perm_n;     // int32 column permutation
    uint64_t md_off, md_n;         // fp16 min scale per superblock
    uint64_t mq_off, mq_n;         // min field per group (biased)
    uint64_t codes_off[SSF_MAX_LEVELS];
    uint64_t codes_n[SSF_MAX_LEVELS];
    uint32_t layout, nbits;
} ssf_rec;

typedef struct {
    char     magic[4];
    uint32_t version;
    uint32_t n_layer, n_embd, n_head, n_head_kv, n_ff, n_vocab, n_ctx_train;
    float    rope_theta, rms_eps;
    uint32_t group, n_levels;
    uint32_t level_bits[SSF_MAX_LEVELS];
    uint64_t n_tensors;
    uint64_t table_off, json_off, json_n, tok_off, tok_n;
    uint64_t group_off;
    uint32_t norm_type, rope_type;
    float    attn_scale, logit_softcap;
    uint32_t n_swa, arch_bits;
    uint32_t n_rot, flags;
    float    emb_scale, res_scale, logit_scale;
    uint32_t n_expert_used, moe_flags;
    float    attn_softcap, clip_qkv;
    float    moe_scale;
    uint32_t moe_groups, moe_topk_group;
    uint32_t ssm_groups, ssm_dstate, ssm_norm_group;
    float    ssm_dt_lo, ssm_dt_hi;
    float    ssm_bcdt_eps;
    uint32_t gdn_nk, gdn_dk;
} ssf_hdr;
#pragma pack(pop)

// Sizes fixed by the format (REC_FMT is 248 bytes, HEADER_FMT 228).
#ifdef __cplusplus
static_assert(sizeof(ssf_rec) == 248, "ssf_rec layout");
static_assert(sizeof(ssf_hdr) == 228, "ssf_hdr layout");
#else
_Static_assert(sizeof(ssf_rec) == 248, "ssf_rec layout");
_Static_assert(sizeof(ssf_hdr) == 228, "ssf_hdr layout");
#endif

typedef struct {
    const uint8_t * base;
    size_t          size;
    const ssf_hdr * hdr;
    const ssf_rec * recs;
    int             scale6, minneg;
} ssf_file;

// Maps `path` read-only and validates the header and every record's ranges.
// Returns 1, or 0 with a reason in why.
int  ssf_open(ssf_file * f, const char * path, char * why, int nwhy);
void ssf_close(ssf_file * f);
const ssf_rec * ssf_find(const ssf_file * f, const char * name);
const ssf_rec * ssf_findf(const ssf_file * f, const char * fmt, int a, int b);

// Bytes of one row of a per-group field array (8-bit: ng, 6-bit: ng/4*3).
static inline size_t ssf_field_row_bytes(int ng, int six) {
    return six ? (size_t) (ng / 4) * 3 : (size_t) ng;
}
static inline int ssf_nscale(int n) { return (n / SSF_GROUP + SSF_GPS - 1) / SSF_GPS; }

// Code planes of a FLAT tensor of width `nbits`, lowest bits first, as the
// format stores them (tooling/sml_quantize.py:106 FLAT_PLANES). Q6 is the one
// width whose planes are not in bit order: plane 0 holds bits 4-5 (2-bit
// group-planar), plane 1 bits 0-3 (nibbles).
//   plane kinds: 4 = nibble plane, 2 = group-planar 2-bit, 1 = bit plane
int ssf_planes(int nbits, int kinds[3], int shifts[3]);

#ifdef __cplusplus
}
#endif
