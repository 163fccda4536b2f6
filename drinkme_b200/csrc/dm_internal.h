// Internal declarations shared by the host layout code, the kernels and the
// C ABI of libdrinkme_b200.so.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/drinkme_b200.h"

namespace dm {

// Rows per unit: a unit is 16 consecutive rows x one block column, the work
// item of the GEMV kernels and the granularity of the device layout. Sixteen
// rows are the m = 16 side of one m16n8k16 MMA (the weights are its A
// operand, the activations its n = 8 B operand).
constexpr int kUnitRows = 16;
// Bytes of a unit's header: per row slot {u16 off16, u16 nesc, u16 sched,
// u16 words}, then the sip exponent tables of the unit's part (4 words).
constexpr int kUnitHeader = kUnitRows * 8 + 16;
// Activations staged per unit: one 1024-weight block column of every
// virtual activation row, row stride 2048 + 16 bytes (an odd number of
// 16-byte slots, so the 8-lane phases of the B-fragment loads do not
// collide on shared-memory banks).
constexpr int kXRowStride = 2048 + 16;
constexpr int kMaxVirtualRows = 8;

struct RowEntry {
    uint16_t off16;  // row-block stream start, in 16-byte units from the unit start
    uint16_t nesc;   // sip fast path: escapes (tier-0 code 7) in the block; else 0
    uint16_t sched;  // >= 3 tiers: the reference's per-block schedule (radix_pack.schedule_np)
    uint16_t words;  // the block's word count in the pack (0: absent row)
};
static_assert(sizeof(RowEntry) == 8, "row entry is 8 bytes");

// One pack (or row shard of a pack) of a tensor: host arrays and shape.
struct PackPart {
    const uint8_t *palette;
    size_t npal;
    const uint32_t *offsets;
    size_t noff;
    const uint32_t *data;
    size_t nwords;
    int64_t R, C;
    const int32_t *widths;
    int32_t nw, B;
    int64_t row0, row1;
};

struct TensorLayout {
    int64_t R = 0, C = 0, row0 = 0, rows = 0;
    int32_t nparts = 1;
    // the packs' own profile when the loader re-encoded them as sip (0: as given)
    int32_t src_nw = 0, src_widths[8] = {0};
    int32_t B = 0, nw = 0, widths[8] = {0};
    int32_t covered = 0;
    uint8_t palette[256] = {0};
    int64_t NB = 0, tiles = 0, units = 0;
    int64_t payload_words = 0;  // NW of this shard
    int64_t read_bytes = 0;      // radix_ops.read_bytes of the source pack(s)
    int64_t dev_read_bytes = 0;  // the same count over the layout the kernels stream
    bool fast_sip = false;
    int32_t max_unit_bytes = 0;
    // padded palette words (radix_pack.padded_palette_words): nonterminal tiers,
    // each (1 << w) - 1 bytes zero-padded to whole words
    uint32_t pal_words[24] = {0};
    int32_t npal_words = 0;
    // per-tier word offset of each tier's table inside pal_words
    int32_t tier_table[8] = {0};
    // sip: the first eight parts' exponent tables (th0, th1, tl0, tl1), as the unit headers hold them
    uint32_t part_tabs[8][4] = {{0}};
};

// Launch knobs of the sip kernels (dm_tensor_set_launch): negative or zero
// fields take the measured defaults.
constexpr int32_t kSplitAuto = 0, kSplitStreamK = 1, kSplitTiles = 2;
struct LaunchKnobs {
    int32_t slots = 0;      // staging slots of the unit ring (0: the measured rule; 1..6)
    int32_t split = kSplitAuto;
    int32_t skew = -1;      // stream-K: units fewer than the average for the last CTA (-1: 4)
    int32_t resident = -1;  // most block columns with resident activations (-1: 16; 0: never)
    int32_t prefetch = -1;  // units each CTA asks into L2 before its dependency wait (-1: 0, none)
};

struct Scratch {
    float *partials = nullptr;   // [max_workers][2][128]: a CTA's sums of its first / last tile
    int *counters = nullptr;     // [tiles] arrival counters, zero between calls
    uint16_t *xsplit = nullptr;  // [6][C] bf16: an fp32 activation pair's hi/mid/lo rows, or up to six
                                 // bf16 rows copied to a 16-byte boundary
    int *err = nullptr;          // device error word
    int32_t max_workers = 0;
};

}  // namespace dm

struct dm_tensor {
    int32_t device = 0;
    dm::TensorLayout L;
    uint8_t *d_data = nullptr;     // unit-major layout + tail pad
    size_t data_bytes = 0;
    uint32_t *d_unit16 = nullptr;  // [units + 1] unit starts in 16-byte units
    uint32_t *d_rowdir = nullptr;  // sip: [16-row padded rows][NB][2] stream offset (16-byte units),
                                   // nesc | part << 11 | escape-index offset (16-byte units) << 16
    size_t rowdir_bytes = 0;
    dm::Scratch S;
    dm::LaunchKnobs K;
    int32_t sms = 148;
    size_t resident_bytes = 0;
};

namespace dm {

void set_error(char *err, size_t len, const std::string &msg);

// Host layout (layout.cpp)
int validate_pack(const uint8_t *palette, size_t npal, const uint32_t *offsets, size_t noff, size_t nwords,
                  int64_t R, int64_t C, const int32_t *widths, int32_t nw, int32_t B, std::string &msg);
int build_layout(const PackPart *parts, int nparts, TensorLayout &L, std::string &bytes, std::string &unit16,
                 std::string &msg, std::string *rowdir = nullptr);
int launch_decode_sip(const dm_tensor *t, uint16_t *out, void *stream, std::string &msg);
void decode_rows(const PackPart &P, uint16_t *out);
int64_t prefill_workspace_bytes(const dm_tensor *t, int64_t M);
int launch_prefill_sip(const dm_tensor *t, const uint16_t *x, int64_t M, const uint16_t *bias, void *out,
                       int out_f32, uint8_t *work, int64_t work_bytes, void *stream, std::string &msg);
int64_t pack_read_bytes(const PackPart &P, int64_t *payload_words);
int64_t block_words_most(int64_t n, const int32_t *widths, int32_t nw);

// Pack encoder (encode.cpp): the parameter checks of radix.pack_array, and
// the palette (exponents by frequency, ties to the lower exponent) with each
// exponent's rank (covered when it is not in the palette).
int check_pack_params(int64_t R, int64_t C, const int32_t *widths, int32_t nw, int32_t B, int32_t *covered,
                      std::string &msg);
void palette_from_histogram(const uint64_t *hist, int32_t covered, uint8_t *palette_out, uint16_t *rank);

// Kernel launchers (kernels.cu)
int launch_decode_generic(const dm_tensor *t, uint16_t *out, void *stream, std::string &msg);
int launch_decode_pack(const uint8_t *palette, size_t npal, int64_t R, int64_t C, const int32_t *widths, int32_t nw,
                       int32_t B, const uint32_t *words, const uint32_t *offsets, uint16_t *out, void *stream,
                       std::string &msg);
int launch_gemv_generic(const dm_tensor *t, const void *x, int x_f32, int64_t M, const uint16_t *bias, void *out,
                        int out_f32, void *stream, std::string &msg);
int launch_gemv_sip(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                    const uint16_t *bias, void *out, int out_f32, void *stream, std::string &msg);
int launch_split_f32(const float *x, int64_t C, int64_t M, uint16_t *out, void *stream, std::string &msg);
int launch_copy_u16(const uint16_t *src, int64_t n, uint16_t *dst, void *stream, std::string &msg);
int gemv_sip_rows(const dm_tensor *t, const void *x, int x_f32, int64_t M, const uint16_t *bias, void *out,
                  int out_f32, uint16_t *xbuf, int64_t xcap, float *partials, int *counters, int64_t max_workers,
                  void *stream, std::string &msg);
int launch_prepare_schedule(const uint32_t *data, size_t nwords, const uint32_t *offsets, int64_t C,
                            const int32_t *widths, int32_t nw, int32_t B, int64_t nblocks, uint16_t *out,
                            void *stream, std::string &msg);
int launch_gemv_raw(const void *w, int64_t R, int64_t C, const void *x, int x_f32, int64_t M, const uint16_t *bias,
                    void *out, int out_f32, void *stream, std::string &msg);
int sip_shared_bytes(const dm_tensor *t, int Mv, int slots, int max_res, int *slot_bytes, int *nslots,
                     int *xres_bytes, int dir_cap, int reserve = 0);
int gemv_plan(const dm_tensor *t, int Mv, dm_launch_plan *out, std::string &msg);
int launch_gemv_sip_with(const dm_tensor *t, const uint16_t *xv, int64_t x_stride, int Mv, int nsplit, int M_out,
                         const uint16_t *bias, void *out, int out_f32, float *partials, int *counters, int *err,
                         int64_t max_workers, void *stream, std::string &msg,
                         const dm_gather *gather = nullptr);

}  // namespace dm
