// prompt.cpp — TTS prompt rows from text (host), declared in include/z2b.h.
//
// Replaces zonos2_build_prompt (src/zonos2-prompt.cpp:54-133, src/zonos2.h:181-195): the rows
// a server admits into a decode step as a new stream's prompt. Each row is n_codebooks audio
// ids + one text id; every audio id is the pad id except in the silence frames.
//
// Text ids: PAD/UNK/BOS/EOS are 0..3, then 192 legacy symbols, then the 256 UTF-8 byte values
// (byte b -> id b + 192). The conditioning ids occupy the top of the text vocabulary, in this
// order: speaking rate, the quality features (one range per feature), speaker background,
// accurate mode; text_vocab itself is the text pad. The conditioning layout is the
// reference's fixed hyper-parameter set (src/zonos2.h:41-46), not a GGUF key.
#include "runtime.h"

#include <algorithm>
#include <cstring>
#include <vector>

namespace {

constexpr int kBos = 2, kEos = 3, kByteBase = 192;
constexpr int kRateBuckets = 8, kBgBuckets = 2, kAccurateBuckets = 1;
constexpr int kQualityCounts[6] = {12, 12, 12, 8, 8, 8};
constexpr int kDefaultQualityFeature = 5, kDefaultQualityBucket = 3;   // trailing_silence_s

// 0.2 s of DAC silence (17 frames x 9 codebooks), the reference's precomputed codes: frame 0,
// frame 1, fourteen copies of one frame, frame 16.
constexpr int kSilenceFrames = 17;
constexpr int32_t kSilenceDistinct[4][9] = {
    {568, 778, 338, 524, 967, 360, 728, 550, 90},
    {568, 778, 10, 674, 364, 981, 741, 378, 731},
    {568, 804, 10, 674, 364, 981, 568, 378, 731},
    {568, 778, 721, 842, 264, 974, 989, 507, 308},
};
int silence_code(int frame, int cb) {
    const int r = frame == 0 ? 0 : frame == 1 ? 1 : frame == kSilenceFrames - 1 ? 3 : 2;
    return kSilenceDistinct[r][cb];
}

}  // namespace

extern "C" {

void z2b_prompt_options_default(z2b_prompt_options* opt) {
    if (!opt) return;
    std::memset(opt, 0, sizeof(*opt));
    opt->prepend_silence = 1;
    opt->speaking_rate_bucket = -1;
    opt->n_quality = 0;
    for (int& q : opt->quality_buckets) q = -1;
    opt->add_speaker_slot = 0;
    opt->clean_speaker_background = 1;
    opt->accurate_mode = 1;
}

int z2b_build_prompt(const z2b_hparams* hp, const char* text, int64_t text_len, const z2b_prompt_options* opt,
                     int32_t* out_ids, int cap_rows, int* n_rows, int* spk_pos) {
    using z2b::set_error;
    if (!hp || !opt || !n_rows || !spk_pos || text_len < 0 || (text_len > 0 && !text)) {
        set_error("null argument");
        return Z2B_ERR_ARG;
    }
    if (opt->n_quality < 0 || opt->n_quality > 16) { set_error("n_quality must be in [0, 16]"); return Z2B_ERR_ARG; }
    if (text_len > (1 << 28)) { set_error("text too long"); return Z2B_ERR_ARG; }
    const int ncb = (int)hp->n_codebooks, W = ncb + 1, pad = (int)hp->audio_pad_id, tv = (int)hp->text_vocab;
    const int n_feat = (int)(sizeof(kQualityCounts) / sizeof(kQualityCounts[0]));
    int sum_q = 0;
    for (int c : kQualityCounts) sum_q += c;
    const int base = tv - kRateBuckets - sum_q - kBgBuckets - kAccurateBuckets;   // first conditioning id
    const int bg_base = base + kRateBuckets + sum_q;

    // text ids of the rows before the text
    std::vector<int> head;
    *spk_pos = -1;
    if (opt->add_speaker_slot) {
        *spk_pos = 0;
        head.push_back(tv);                                   // the speaker slot
        if (kBgBuckets > 0) {
            head.push_back(bg_base + (opt->clean_speaker_background ? 0 : 1));
            if (kAccurateBuckets > 0 && opt->accurate_mode) head.push_back(bg_base + kBgBuckets);
        }
    }
    if (opt->speaking_rate_bucket >= 0) head.push_back(base + opt->speaking_rate_bucket);
    int qb[16];
    int nq = opt->n_quality;
    if (nq == 0) {
        nq = n_feat;
        for (int f = 0; f < n_feat; ++f) qb[f] = f == kDefaultQualityFeature ? kDefaultQualityBucket : -1;
    } else {
        std::memcpy(qb, opt->quality_buckets, sizeof(int) * nq);
    }
    for (int f = 0, prefix = 0; f < n_feat; prefix += kQualityCounts[f], ++f)
        if (f < nq && qb[f] >= 0) head.push_back(base + kRateBuckets + prefix + qb[f]);

    const int64_t rows = (int64_t)head.size() + 2 + text_len + (opt->prepend_silence ? kSilenceFrames : 0);
    *n_rows = (int)rows;
    if (cap_rows < rows || !out_ids) {
        if (cap_rows == 0 && !out_ids) return Z2B_OK;         // sizing call
        set_error("out_ids holds fewer rows than the prompt");
        return Z2B_ERR_ARG;
    }
    int32_t* o = out_ids;
    auto text_row = [&](int t) {
        for (int c = 0; c < ncb; ++c) o[c] = pad;
        o[ncb] = t;
        o += W;
    };
    for (int t : head) text_row(t);
    text_row(kBos);
    for (int64_t i = 0; i < text_len; ++i) text_row(kByteBase + (int)(unsigned char)text[i]);
    text_row(kEos);
    if (opt->prepend_silence) {
        // delayed (sheared) codebooks: codebook c of row t is silence frame t - c
        for (int t = 0; t < kSilenceFrames; ++t) {
            for (int c = 0; c < ncb; ++c) o[c] = (c < 9 && t >= c) ? silence_code(t - c, c) : pad;
            o[ncb] = tv;
            o += W;
        }
    }
    return Z2B_OK;
}

}  // extern "C"
