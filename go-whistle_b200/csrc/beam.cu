// beam.cu — internal/search's beam search (search/beam.go, options.go) over
// the device decoder, for many clips at once.
//
// Every hypothesis of clip c holds one of the clip's `beams` decoder
// streams [c·beams, (c+1)·beams): the stream whose state has consumed the
// hypothesis' sequence but its last token. A step feeds every live
// hypothesis its last token on its stream — one decoder step for all
// streams of all clips (a CUDA graph), the exact head, then the n best next
// tokens and the float64 log-sum-exp of each live stream's logits on the
// device — and runs beam.go's bookkeeping on the host. Children that share
// a parent's stream get streams of their own before the next step by a
// fork (decoder.go:223 State.Fork, beam.go:537 own): the parent's state is
// copied on the device into a stream no live hypothesis holds. All
// hypotheses of a search advance in lockstep, one position per step, so
// every stream sits at the same position.
//
// The ranking arithmetic is the reference's, in float64: log p = x − lse,
// summed log p over the length penalty (options.go:213), stable sorts
// that keep the parent's rank, then the candidate's, on ties.
#include <algorithm>
#include <cmath>
#include <limits>
#include <vector>

#include "common.cuh"
#include "decoder_beam.cuh"

using namespace wb;

namespace {

struct Cand {
    int tok;
    double lp, adj;  // the model's log p; after Adjust (none here: equal)
};

struct Hyp {
    std::vector<int32_t> text;  // text tokens (without EOS)
    std::vector<double> lps;    // log p of each text token, then of EOS
    int lang = -1;
    double lang_lp = 0.0, sum = 0.0, adj = 0.0;
    bool eos = false;
    int stream = -1;  // the decoder stream holding its state
    int feed = -1;    // the token its stream has not consumed yet
};

struct Clip {
    std::vector<Hyp> alive, fin;
    bool done = false;
};

struct Search {
    wc_beam_options o;
    int eos;
    static constexpr int kPrompt = 1;  // the prompt is [bos]

    // options.go:213 penalty.
    double penalty(int l) const {
        switch (o.norm) {
        case WC_NORM_LEN:
            return (double)std::max(l, 1);
        case WC_NORM_POW:
            return std::pow((double)std::max(l, 1), o.alpha);
        case WC_NORM_GNMT:
            return std::pow((5.0 + (double)l) / 6.0, o.alpha);
        default:
            return 1.0;
        }
    }
    // beam.go:209 length.
    int length(const Hyp &h) const {
        int l = (int)h.text.size();
        if (o.length == WC_LEN_SEQ) l = kPrompt + 1 + l;
        if (h.eos && o.length != WC_LEN_TEXT) l++;
        return l;
    }
    double score(const Hyp &h) const { return h.adj / penalty(length(h)); }

    Hyp child(const Hyp &h, const Cand &c) const {
        Hyp k;
        k.text = h.text;
        k.lps = h.lps;
        k.lps.push_back(c.lp);
        k.lang = h.lang;
        k.lang_lp = h.lang_lp;
        k.sum = h.sum + c.lp;
        k.adj = h.adj + c.adj;
        k.stream = h.stream;
        if (c.tok == eos) {
            k.eos = true;
        } else {
            k.text.push_back(c.tok);
            k.feed = c.tok;
        }
        return k;
    }

    // beam.go:436 worst: the first finished hypothesis of the lowest score.
    size_t worst(const Clip &c) const {
        size_t w = 0;
        for (size_t i = 0; i < c.fin.size(); i++)
            if (score(c.fin[i]) < score(c.fin[w])) w = i;
        return w;
    }

    // beam.go:381 finish, 399 finishK (Whisper's finished-hypothesis rule).
    void finish(Clip &c, Hyp &&h) const {
        const size_t k = (size_t)o.beams;
        switch (o.stop) {
        case WC_STOP_K:
            if (c.fin.size() < k) c.fin.push_back(std::move(h));
            break;
        case WC_STOP_HF:
            c.fin.push_back(std::move(h));
            if (c.fin.size() > k) c.fin.erase(c.fin.begin() + (long)worst(c));
            break;
        default:
            c.fin.push_back(std::move(h));
        }
    }

    // beam.go:449 done.
    bool done(const Clip &c) const {
        if (c.alive.empty()) return true;
        if (c.fin.empty()) return false;
        double live = -std::numeric_limits<double>::infinity();
        for (const Hyp &h : c.alive) live = std::max(live, score(h));
        switch (o.stop) {
        case WC_STOP_K:
            return c.fin.size() >= (size_t)o.beams;
        case WC_STOP_BEST: {
            double best = -std::numeric_limits<double>::infinity();
            for (const Hyp &h : c.fin) best = std::max(best, score(h));
            return best >= live;
        }
        case WC_STOP_HF: {
            if (c.fin.size() < (size_t)o.beams) return false;
            double w = std::numeric_limits<double>::infinity();
            for (const Hyp &h : c.fin) w = std::min(w, score(h));
            return w >= live;
        }
        }
        return false;
    }

    // beam.go:247 step on the candidates of the clip's live hypotheses
    // (cands[i]: the best n of alive[i], best first).
    void step(Clip &c, const std::vector<std::vector<Cand>> &cands) const {
        const int k = o.beams;
        std::vector<Hyp> kids;
        for (size_t i = 0; i < c.alive.size(); i++)
            for (size_t j = 0; j < cands[i].size(); j++) {
                if ((int)j > k && cands[i][j].tok == eos) continue;
                kids.push_back(child(c.alive[i], cands[i][j]));
            }
        std::stable_sort(kids.begin(), kids.end(), [](const Hyp &a, const Hyp &b) { return a.adj > b.adj; });
        if (o.stop == WC_STOP_ALL) {
            std::vector<Hyp> pool = std::move(c.fin);
            for (Hyp &h : kids) pool.push_back(std::move(h));
            std::stable_sort(pool.begin(), pool.end(),
                             [this](const Hyp &a, const Hyp &b) { return score(a) > score(b); });
            c.fin.clear();
            c.alive.clear();
            for (size_t i = 0; i < pool.size() && i < (size_t)k; i++)
                (pool[i].eos ? c.fin : c.alive).push_back(std::move(pool[i]));
            c.done = c.alive.empty();
            return;
        }
        c.alive.clear();
        for (size_t rank = 0; rank < kids.size(); rank++) {
            Hyp &h = kids[rank];
            if (!h.eos) {
                c.alive.push_back(std::move(h));
                if ((int)c.alive.size() == k) break;
                continue;
            }
            if (o.admit == WC_ADMIT_TOPK && (int)rank >= k) continue;
            finish(c, std::move(h));
        }
        c.done = done(c);
    }

    // beam.go:113 pick: the best final score among the finished, with the
    // live ones competing unless the stopping rule ended the search.
    const Hyp *pick(const Clip &c) const {
        std::vector<const Hyp *> pool;
        for (const Hyp &h : c.fin) pool.push_back(&h);
        if (!c.done || pool.empty()) {
            std::vector<const Hyp *> live;
            for (const Hyp &h : c.alive) live.push_back(&h);
            if (o.stop == WC_STOP_K) {
                std::stable_sort(live.begin(), live.end(), [](const Hyp *a, const Hyp *b) { return a->adj > b->adj; });
                const long keep = std::max<long>((long)o.beams - (long)pool.size(), 0);
                if ((long)live.size() > keep) live.resize((size_t)keep);
            }
            pool.insert(pool.end(), live.begin(), live.end());
        }
        const Hyp *best = nullptr;
        for (const Hyp *h : pool)
            if (!best || score(*h) > score(*best)) best = h;
        return best;
    }
};

// beam.go:537 own: every live hypothesis gets a stream of its own; the
// first holder of a shared stream keeps it, the others take streams of the
// clip that no live hypothesis holds, with a fork of the shared state.
void own(std::vector<Clip> &clips, int beams, std::vector<int32_t> &pairs) {
    for (size_t ci = 0; ci < clips.size(); ci++) {
        Clip &c = clips[ci];
        if (c.done) continue;
        const int base = (int)ci * beams;
        std::vector<char> held(beams, 0), kept(beams, 0);
        for (const Hyp &h : c.alive) held[h.stream - base] = 1;
        int next_free = 0;
        for (Hyp &h : c.alive) {
            const int s = h.stream - base;
            if (!kept[s]) {
                kept[s] = 1;
                continue;
            }
            while (held[next_free]) next_free++;  // alive.size() <= beams: one exists
            held[next_free] = kept[next_free] = 1;
            pairs.push_back(h.stream);
            pairs.push_back(base + next_free);
            h.stream = base + next_free;
        }
    }
}

}  // namespace

extern "C" void wc_beam_default(wc_beam_options *o) {
    if (!o) return;
    o->beams = 5;
    o->max_tokens = 0;
    o->language = -1;
    o->norm = WC_NORM_LEN;
    o->alpha = 1.0;
    o->length = WC_LEN_TEXT;
    o->stop = WC_STOP_K;
    o->admit = WC_ADMIT_ABOVE_LIVE;
    o->lang_step = WC_LANG_ARGMAX;
}

// options.go:160 Validate.
static wc_status validate(const wc_beam_options &o) {
    const char *bad = "search: invalid options";
    if (o.beams < 1 || o.beams > 63) return set_error(WC_ERR_INVALID, fmt("%s: %d beams", bad, o.beams));
    if (o.max_tokens < 0) return set_error(WC_ERR_INVALID, fmt("%s: max tokens %d", bad, o.max_tokens));
    if (o.norm < WC_NORM_NONE || o.norm > WC_NORM_GNMT) return set_error(WC_ERR_INVALID, fmt("%s: norm %d", bad, o.norm));
    if (o.length < WC_LEN_TEXT || o.length > WC_LEN_SEQ)
        return set_error(WC_ERR_INVALID, fmt("%s: length %d", bad, o.length));
    if (o.stop < WC_STOP_ALL || o.stop > WC_STOP_HF) return set_error(WC_ERR_INVALID, fmt("%s: stop %d", bad, o.stop));
    if (o.admit < WC_ADMIT_TOPK || o.admit > WC_ADMIT_ABOVE_LIVE)
        return set_error(WC_ERR_INVALID, fmt("%s: admit %d", bad, o.admit));
    if (o.lang_step < WC_LANG_ARGMAX || o.lang_step > WC_LANG_BEAM)
        return set_error(WC_ERR_INVALID, fmt("%s: language step %d", bad, o.lang_step));
    if (std::isnan(o.alpha) || std::isinf(o.alpha)) return set_error(WC_ERR_INVALID, fmt("%s: alpha %g", bad, o.alpha));
    return WC_OK;
}

#define BEAM_ST(call)                \
    do {                             \
        wc_status s_ = (call);       \
        if (s_ != WC_OK) return s_;  \
    } while (0)

extern "C" wc_status wc_decoder_beam(wc_decoder *d, const wc_beam_options *opt, int bos, const int32_t *langs,
                                     int n_langs, int eos, int32_t *tokens, int32_t *counts, int32_t *lang,
                                     int32_t *eos_hit, double *score, double *lang_logprob, double *logprobs,
                                     wc_stream stream) {
    if (!opt) return set_error(WC_ERR_INVALID, "search: nil options");
    BEAM_ST(validate(*opt));
    DecBeamInfo info{};
    BEAM_ST(dec_beam_info(d, &info));
    const int B = opt->beams;
    if (info.group != B)
        return set_error(WC_ERR_INVALID, fmt("search: the memory holds %d streams per clip, the options %d beams",
                                             info.group, B));
    if (info.len != 0)
        return set_error(WC_ERR_INVALID, fmt("search: the streams are at position %d (call wc_decoder_memory_beams)",
                                             info.len));
    if (!langs || n_langs <= 0 || n_langs > 64 || !tokens || !counts || !lang || !eos_hit || !score)
        return set_error(WC_ERR_INVALID, fmt("search: beam search with %d languages", n_langs));
    if (opt->language < -1 || opt->language >= n_langs)
        return set_error(WC_ERR_INVALID, fmt("search: unknown language %d of %d", opt->language, n_langs));
    if (bos < 0 || bos >= info.vocab || eos < 0 || eos >= info.vocab)
        return set_error(WC_ERR_INVALID, fmt("search: token %d out of range [0, %d)",
                                             bos < 0 || bos >= info.vocab ? bos : eos, info.vocab));
    for (int i = 0; i < n_langs; i++)
        if (langs[i] < 0 || langs[i] >= info.vocab)
            return set_error(WC_ERR_INVALID, fmt("search: token %d out of range [0, %d)", langs[i], info.vocab));
    const int max_tok = opt->max_tokens > 0 ? opt->max_tokens : info.positions;
    if (max_tok > info.positions)
        return set_error(WC_ERR_INVALID, fmt("search: %d positions exceed the decoder's %d", max_tok, info.positions));
    if (B + 1 > info.vocab) return set_error(WC_ERR_INVALID, fmt("search: %d beams over %d tokens", B, info.vocab));
    cudaStream_t st = (cudaStream_t)stream;
    const int S = info.streams, C = S / B;
    Search srch{*opt, eos};
    std::vector<Clip> clips((size_t)C);
    std::vector<int32_t> feed((size_t)S, bos), rows, ctok, pairs;
    std::vector<float> clogit;
    std::vector<double> clse;

    // beam.go:144 languageStep: the prompt on each clip's first stream,
    // then the n best of the (forced or all) language tokens.
    std::vector<int32_t> ids;
    if (opt->language >= 0)
        ids.push_back(langs[opt->language]);
    else
        ids.assign(langs, langs + n_langs);
    const int nl = opt->lang_step == WC_LANG_BEAM ? std::min(B, (int)ids.size()) : 1;
    BEAM_ST(dec_beam_feed(d, feed.data(), st));
    for (int c = 0; c < C; c++) rows.push_back(c * B);
    ctok.resize((size_t)C * nl);
    clogit.resize(ctok.size());
    clse.resize((size_t)C);
    BEAM_ST(dec_beam_top(d, rows.data(), C, nl, ids.data(), (int)ids.size(), ctok.data(), clogit.data(), clse.data(),
                         st));
    const bool scored = opt->lang_step != WC_LANG_ARGMAX && opt->language < 0;
    for (int c = 0; c < C; c++)
        for (int j = 0; j < nl; j++) {
            Hyp h;
            h.lang = ctok[(size_t)c * nl + j];
            h.lang_lp = (double)clogit[(size_t)c * nl + j] - clse[c];
            if (scored) h.sum = h.adj = h.lang_lp;
            h.stream = c * B;
            h.feed = h.lang;
            clips[c].alive.push_back(std::move(h));
        }

    const int n = B + 1;  // Whisper's k + 1 candidates per parent
    for (int step = 0; step < max_tok - 1; step++) {
        bool any = false;
        for (const Clip &c : clips) any |= !c.done;
        if (!any) break;
        pairs.clear();
        own(clips, B, pairs);
        BEAM_ST(dec_beam_fork(d, pairs.data(), (int)pairs.size() / 2, st));
        std::fill(feed.begin(), feed.end(), eos);
        rows.clear();
        for (const Clip &c : clips) {
            if (c.done) continue;
            for (const Hyp &h : c.alive) {
                feed[h.stream] = h.feed;
                rows.push_back(h.stream);
            }
        }
        BEAM_ST(dec_beam_feed(d, feed.data(), st));
        const size_t nr = rows.size();
        ctok.resize(nr * n);
        clogit.resize(nr * n);
        clse.resize(nr);
        BEAM_ST(dec_beam_top(d, rows.data(), (int)nr, n, nullptr, 0, ctok.data(), clogit.data(), clse.data(), st));
        size_t r = 0;
        for (Clip &c : clips) {
            if (c.done) continue;
            std::vector<std::vector<Cand>> cands(c.alive.size());
            for (size_t i = 0; i < c.alive.size(); i++, r++)
                for (int j = 0; j < n; j++) {
                    const double lp = (double)clogit[r * n + j] - clse[r];
                    cands[i].push_back({ctok[r * n + j], lp, lp});
                }
            srch.step(c, cands);
        }
    }

    const int out_w = max_tok > 1 ? max_tok - 1 : 1;
    for (int c = 0; c < C; c++) {
        const Hyp *h = srch.pick(clips[c]);
        int32_t *row = tokens + (size_t)c * out_w;
        std::fill(row, row + out_w, -1);
        if (logprobs) std::fill(logprobs + (size_t)c * max_tok, logprobs + (size_t)(c + 1) * max_tok, 0.0);
        if (!h) {
            counts[c] = 0, lang[c] = -1, eos_hit[c] = 0, score[c] = -std::numeric_limits<double>::infinity();
            if (lang_logprob) lang_logprob[c] = 0.0;
            continue;
        }
        const size_t nt = std::min(h->text.size(), (size_t)out_w);
        std::copy(h->text.begin(), h->text.begin() + (long)nt, row);
        counts[c] = (int32_t)nt;
        lang[c] = h->lang;
        eos_hit[c] = h->eos ? 1 : 0;
        score[c] = srch.score(*h);
        if (lang_logprob) lang_logprob[c] = h->lang_lp;
        if (logprobs)
            std::copy(h->lps.begin(), h->lps.begin() + (long)std::min(h->lps.size(), (size_t)max_tok),
                      logprobs + (size_t)c * max_tok);
    }
    return WC_OK;
}
