// Continuous-batching engine over the d1h runners: a C++ restatement of src/engine.rs:149-525 (Engine::admit /
// run / process_media / encode_group / launch_batch / complete / finish_job). One engine owns one device's text
// model, workspace, optional vision / audio encoders and one stream; the caller drives it (d1e_step) from one host
// thread, so a multi-GPU server runs one engine per device on its own thread and a dispatcher hands whole requests
// to the device with the fewest queued tokens (requests are independent; nothing crosses devices).
//
// Per iteration (src/engine.rs:182-221): a text batch is packed FIFO across requests under the token budget and
// launched, then at most one media group (images of several requests share one vision pass; all prefixes of the
// group share one trunk prefix pass) is encoded; up to two batches stay in flight so the host work of batch N+1
// overlaps the GPU work of batch N; finished batches hand their logits back to their requests.
//
// Differences from the reference, both B200-side: the audio clips of a media group are encoded in one packed
// d1h_audio_encode call (the reference encodes clip by clip), and a finished request's logits wait in a completion
// queue for d1e_take instead of being sent on a channel.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <deque>
#include <map>
#include <string>
#include <vector>

#include "d1h.h"

namespace {

constexpr int ED = 1024;     // src/model.rs:12
constexpr int SLOTS = 2;     // src/model.rs:251
constexpr int KV_DIM = 512;

thread_local std::string e_err;

int efail(const std::string& m, int code = -1) {
    e_err = m;
    return code;
}

// Encoder rows of an audio clip of `valid` mel frames: three stride-2 stages (src/engine.rs:36-42).
size_t audio_rows(int valid) {
    size_t l = valid;
    for (int i = 0; i < 3; i++) l = (l - 1) / 2 + 1;
    return l;
}

struct Row {
    std::vector<int> ids, markers;
    int qtype = 0;
};

struct JobState {
    long long id = 0;
    std::vector<Row> rows;
    int kind = 0;                        // D1_MEDIA_NONE / IMAGES / AUDIO
    std::vector<int> ph, pw;             // image crops
    std::vector<uint16_t> patches;       // fp16 bits [sum ph*pw][768]
    std::vector<float> mel;              // audio [valid][128] log-mel frames, or
    std::vector<float> pcm;              // audio as a waveform at `rate` Hz
    int rate = 16000;
    int valid = 0;
    bool has_prefix = false;
    D1PrefixCache prefix{};
    size_t prefix_bytes = 0;
    bool media_done = false;
    size_t next_row = 0, done_rows = 0;
    std::vector<std::vector<float>> results;
    std::string failed;

    size_t prefix_len() const {
        if (kind == D1_MEDIA_IMAGES) {
            size_t t = 0;
            for (size_t i = 0; i < ph.size(); i++) t += (size_t)ph[i] * pw[i] / 4;
            return t;
        }
        if (kind == D1_MEDIA_AUDIO) return audio_rows(valid);
        return 0;
    }
    size_t patches_n() const {
        size_t t = 0;
        for (size_t i = 0; i < ph.size(); i++) t += (size_t)ph[i] * pw[i];
        return t;
    }
};

struct InFlight {
    int slot = -1;                                    // -1: a prefix pass (nothing to collect)
    std::vector<std::tuple<long long, size_t, int>> rows;  // (job, row, n_markers)
};

struct Done {
    long long id;
    std::vector<float> logits;
    std::string err;
};

}  // namespace

struct D1Engine {
    D1Model* m = nullptr;
    D1Vision* vision = nullptr;
    D1Audio* audio = nullptr;
    D1Workspace* ws = nullptr;
    cudaStream_t st = nullptr;
    int device = 0;
    D1EngineConfig cfg{};
    int n_attn = 0, n_conv = 0, vision_patches = 0;
    int cap_markers = 0;
    std::map<long long, JobState> jobs;
    std::deque<long long> order;
    long long next_id = 0;
    std::deque<InFlight> inflight;
    int slot = 0;
    size_t cache_bytes = 0;
    double long_cost = 0, short_cost = 0;
    std::deque<Done> done;
    long long st_tokens = 0, st_batches = 0, st_media = 0, st_media_tokens = 0, st_rows = 0;
    std::vector<float> logit_buf;

    size_t prefix_bytes_for(size_t len) const {  // PrefixCache::bytes_for, src/model.rs:82-84
        return 2 * (size_t)n_attn * len * KV_DIM * 2 + (size_t)n_conv * ED * 2;
    }

    int next_slot() {  // src/engine.rs:223-232
        if ((int)inflight.size() >= SLOTS) {
            InFlight f = inflight.front();
            inflight.pop_front();
            if (complete(f)) return -1;
        }
        const int s = slot;
        slot = (slot + 1) % SLOTS;
        return s;
    }

    void finish_job(long long id) {  // src/engine.rs:512-525
        auto it = jobs.find(id);
        if (it == jobs.end()) return;
        JobState& js = it->second;
        order.erase(std::remove(order.begin(), order.end(), id), order.end());
        if (js.has_prefix) {
            cache_bytes -= js.prefix_bytes;
            d1h_prefix_free(&js.prefix, st);
        }
        Done d{id, {}, js.failed};
        if (js.failed.empty())
            for (auto& r : js.results) d.logits.insert(d.logits.end(), r.begin(), r.end());
        done.push_back(std::move(d));
        jobs.erase(it);
    }

    int complete(const InFlight& f) {  // src/engine.rs:487-510
        if (f.slot < 0) return 0;
        const int n = d1h_finish(m, ws, f.slot, logit_buf.data(), (int)logit_buf.size());
        if (n < 0) return efail(std::string("finish failed: ") + d1h_last_error());
        size_t off = 0;
        std::vector<long long> finished;
        for (const auto& [id, r, nm] : f.rows) {
            auto it = jobs.find(id);
            if (it != jobs.end()) {
                JobState& js = it->second;
                js.results[r].assign(logit_buf.begin() + off, logit_buf.begin() + off + nm);
                if (++js.done_rows == js.rows.size()) finished.push_back(id);
            }
            off += nm;
        }
        for (long long id : finished) finish_job(id);
        return 0;
    }

    // src/engine.rs:252-285: one media group, FIFO within the cache budget, small groups.
    int process_media_limited(int max_groups, bool& any) {
        any = false;
        for (int g = 0; g < max_groups; g++) {
            std::vector<long long> group;
            size_t tokens = 0, patches = 0, bytes = 0;
            for (long long id : order) {
                const JobState& js = jobs.at(id);
                if (js.media_done) continue;
                const size_t p = js.prefix_len();
                const size_t np = js.kind == D1_MEDIA_IMAGES ? js.patches_n() : 0;
                const size_t need = prefix_bytes_for(p) + p * ED * 4;
                if (cache_bytes + bytes + need > (size_t)cfg.media_cache_bytes && cache_bytes + bytes > 0) break;
                const size_t cap_p = vision_patches > 0 ? (size_t)vision_patches : SIZE_MAX;
                if (!group.empty() && (tokens + p > 2048 || patches + np > cap_p || group.size() >= 4))
                    break;
                group.push_back(id);
                tokens += p;
                patches += np;
                bytes += need;
            }
            if (group.empty()) return 0;
            if (encode_group(group)) return -1;
            any = true;
        }
        return 0;
    }

    // src/engine.rs:287-397
    int encode_group(const std::vector<long long>& group) {
        std::vector<std::tuple<long long, size_t, size_t>> ok;  // (job, offset, len)
        size_t total = 0;
        for (long long id : group) {
            JobState& js = jobs.at(id);
            const size_t p = js.prefix_len();
            std::string err;
            if (p == 0 || (int)p > cfg.cap_tokens)
                err = "media prefix of " + std::to_string(p) + " positions exceeds the context";
            else if (js.kind == D1_MEDIA_IMAGES && !vision)
                err = "this engine was created without a vision encoder";
            else if (js.kind == D1_MEDIA_AUDIO && !audio)
                err = "this engine was created without an audio encoder";
            if (!err.empty()) {
                js.failed = err;
                js.media_done = true;
                continue;
            }
            ok.push_back({id, total, p});
            total += p;
        }
        if (ok.empty()) return 0;
        float* emb = nullptr;
        if (cudaMallocAsync((void**)&emb, total * ED * 4, st) != cudaSuccess) return efail("prefix buffer allocation");
        // vision: batch crops across jobs up to the tower capacity (an oversized image is chunked)
        std::vector<int> bph, bpw;
        std::vector<uint16_t> bpix;
        size_t batch_off = 0, batch_patches = 0;
        auto flush = [&](size_t next_off) -> int {
            if (!bph.empty()) {
                if (d1h_vision_encode(vision, (int)bph.size(), bph.data(), bpw.data(),
                                      reinterpret_cast<const d1_half*>(bpix.data()), emb + batch_off * ED, st))
                    return efail(std::string("vision encode failed: ") + d1h_last_error());
            }
            bph.clear();
            bpw.clear();
            bpix.clear();
            batch_off = next_off;
            batch_patches = 0;
            return 0;
        };
        // audio clips of the group go through one packed encoder call per input form (log-mel frames, waveforms),
        // then each clip's rows move to its offset
        std::vector<int> avalid, pvalid, pns, prate;
        std::vector<float> amel, apcm;
        std::vector<size_t> aoff, poff;
        for (const auto& [id, off, len] : ok) {
            const JobState& js = jobs.at(id);
            if (js.kind == D1_MEDIA_IMAGES) {
                size_t out = off, i = 0, pstart = 0;
                while (i < js.ph.size()) {
                    size_t j = i, np = 0;
                    while (j < js.ph.size() && np + (size_t)js.ph[j] * js.pw[j] <= (size_t)vision_patches) {
                        np += (size_t)js.ph[j] * js.pw[j];
                        j++;
                    }
                    if (j == i) return efail("an image crop exceeds the vision batch capacity");
                    if (batch_patches + np > (size_t)vision_patches || (bph.empty() && batch_off != out))
                        if (flush(out)) return -1;
                    size_t tok = 0;
                    for (size_t q = i; q < j; q++) {
                        bph.push_back(js.ph[q]);
                        bpw.push_back(js.pw[q]);
                        tok += (size_t)js.ph[q] * js.pw[q] / 4;
                    }
                    bpix.insert(bpix.end(), js.patches.begin() + pstart * 768, js.patches.begin() + (pstart + np) * 768);
                    pstart += np;
                    out += tok;
                    batch_patches += np;
                    i = j;
                }
            } else if (js.kind == D1_MEDIA_AUDIO) {
                if (flush(off)) return -1;
                if (!js.pcm.empty()) {
                    pvalid.push_back(js.valid);
                    pns.push_back((int)js.pcm.size());
                    prate.push_back(js.rate);
                    apcm.insert(apcm.end(), js.pcm.begin(), js.pcm.end());
                    poff.push_back(off);
                } else {
                    avalid.push_back(js.valid);
                    amel.insert(amel.end(), js.mel.begin(), js.mel.begin() + (size_t)js.valid * 128);
                    aoff.push_back(off);
                }
            }
        }
        if (flush(0)) return -1;
        for (int form = 0; form < 2; form++) {
            const std::vector<int>& vv = form ? pvalid : avalid;
            const std::vector<size_t>& oo = form ? poff : aoff;
            if (vv.empty()) continue;
            size_t arows = 0;
            for (int v : vv) arows += audio_rows(v);
            float* tmp = nullptr;
            if (cudaMallocAsync((void**)&tmp, arows * ED * 4, st) != cudaSuccess) return efail("audio buffer allocation");
            const int r = form ? d1h_audio_encode_pcm_rates(audio, (int)vv.size(), pns.data(), prate.data(), apcm.data(),
                                                            tmp, nullptr, st)
                               : d1h_audio_encode(audio, (int)vv.size(), vv.data(), amel.data(), tmp, st);
            if (r < 0) return efail(std::string("audio encode failed: ") + d1h_last_error());
            size_t src = 0;
            for (size_t c = 0; c < vv.size(); c++) {
                const size_t t = audio_rows(vv[c]);
                if (cudaMemcpyAsync(emb + oo[c] * ED, tmp + src * ED, t * ED * 4, cudaMemcpyDeviceToDevice, st) !=
                    cudaSuccess)
                    return efail("audio prefix copy failed");
                src += t;
            }
            cudaFreeAsync(tmp, st);
        }
        std::vector<D1PrefixCache> caches(ok.size());
        for (size_t i = 0; i < ok.size(); i++)
            if (d1h_prefix_alloc(m, (int)std::get<2>(ok[i]), &caches[i], st))
                return efail(std::string("prefix cache allocation failed: ") + d1h_last_error());
        const int s = next_slot();
        if (s < 0) return -1;
        std::vector<D1PrefixSeq> items(ok.size());
        for (size_t i = 0; i < ok.size(); i++) items[i] = D1PrefixSeq{emb + std::get<1>(ok[i]) * ED, &caches[i]};
        if (d1h_launch_prefix(m, ws, s, items.data(), (int)items.size(), st))
            return efail(std::string("prefix pass failed: ") + d1h_last_error());
        inflight.push_back(InFlight{});
        cudaFreeAsync(emb, st);
        short_cost += 3.0 * (double)total;
        st_media_tokens += (long long)total;
        for (size_t i = 0; i < ok.size(); i++) {
            JobState& js = jobs.at(std::get<0>(ok[i]));
            js.prefix = caches[i];
            js.has_prefix = true;
            js.prefix_bytes = prefix_bytes_for(std::get<2>(ok[i]));
            cache_bytes += js.prefix_bytes;
            js.media_done = true;
            st_media++;
        }
        return 0;
    }

    // src/engine.rs:399-485
    int launch_batch(bool& launched) {
        if (long_cost * 3.0 > short_cost) {
            if (launch_batch_filtered(true, launched)) return -1;
            if (launched) return 0;
        }
        return launch_batch_filtered(false, launched);
    }

    int launch_batch_filtered(bool short_only, bool& launched) {
        launched = false;
        const size_t budget = cfg.max_batch_tokens, lng = std::max<size_t>(budget / 2, 1);
        std::vector<std::pair<long long, size_t>> picked;
        size_t tokens = 0, markers = 0;
        std::vector<long long> failed;
        for (long long id : order) {
            JobState& js = jobs.at(id);
            if (!js.failed.empty()) {
                failed.push_back(id);
                continue;
            }
            if (!js.media_done) continue;
            bool stop = false, skip = false;
            for (size_t r = js.next_row; r < js.rows.size(); r++) {
                const size_t n = js.rows[r].ids.size(), nm = js.rows[r].markers.size();
                if (short_only && n > lng) {
                    skip = true;
                    break;
                }
                if (!picked.empty() && (tokens + n > budget || markers + nm > (size_t)cap_markers)) {
                    stop = true;
                    break;
                }
                if (n > (size_t)cfg.cap_tokens) {
                    failed.push_back(id);
                    skip = true;
                    break;
                }
                picked.push_back({id, r});
                tokens += n;
                markers += nm;
            }
            (void)skip;
            if (stop) break;
        }
        for (long long id : failed) {
            JobState& js = jobs.at(id);
            if (js.failed.empty()) js.failed = "a question exceeds the batch capacity";
            finish_job(id);
        }
        if (picked.empty()) return 0;
        bool has_long = false;
        for (auto& [id, r] : picked) has_long |= jobs.at(id).rows[r].ids.size() > lng;
        (has_long ? long_cost : short_cost) += (double)tokens;
        if (long_cost + short_cost > 4e6) {
            long_cost *= 0.5;
            short_cost *= 0.5;
        }
        const int s = next_slot();
        if (s < 0) return -1;
        InFlight f;
        f.slot = s;
        std::vector<D1TextSeq> seqs;
        seqs.reserve(picked.size());
        for (auto& [id, r] : picked) {
            JobState& js = jobs.at(id);
            const Row& row = js.rows[r];
            seqs.push_back(D1TextSeq{row.ids.data(), (int)row.ids.size(), row.markers.data(), (int)row.markers.size(),
                                     row.qtype, js.has_prefix ? &js.prefix : nullptr});
            f.rows.push_back({id, r, (int)row.markers.size()});
        }
        if (d1h_launch_text(m, ws, s, seqs.data(), (int)seqs.size(), st))
            return efail(std::string("launch_text failed: ") + d1h_last_error());
        for (auto& [id, r] : picked) jobs.at(id).next_row = r + 1;
        st_batches++;
        st_rows += (long long)picked.size();
        st_tokens += (long long)tokens;
        inflight.push_back(std::move(f));
        launched = true;
        return 0;
    }

    // src/engine.rs:182-221 (one iteration; admission happens in d1e_submit)
    int step() {
        const size_t before = done.size();
        bool launched = false, media = false;
        if (launch_batch(launched)) return -1;
        if (process_media_limited(1, media)) return -1;
        if (!launched && !media) {
            if (!inflight.empty()) {
                InFlight f = inflight.front();
                inflight.pop_front();
                if (complete(f)) return -1;
            } else if (!order.empty()) {
                // waiting for media budget with nothing in flight: force one group past the budget
                const long long saved = cfg.media_cache_bytes;
                cfg.media_cache_bytes = (long long)1 << 62;
                bool any = false;
                const int r = process_media_limited(1, any);
                cfg.media_cache_bytes = saved;
                if (r) return -1;
            }
        } else if ((int)inflight.size() >= SLOTS) {
            InFlight f = inflight.front();
            inflight.pop_front();
            if (complete(f)) return -1;
        }
        return (int)(done.size() - before);
    }
};

extern "C" {

D1Engine* d1e_create(D1Model* m, D1Vision* vision, D1Audio* audio, const D1EngineConfig* cfg, cudaStream_t stream) {
    if (!m || !cfg || cfg->max_batch_tokens < 1 || cfg->cap_tokens < 64 || cfg->media_cache_bytes < 0) {
        efail("invalid engine configuration");
        return nullptr;
    }
    D1Engine* e = new D1Engine();
    e->m = m;
    e->vision = vision;
    e->audio = audio;
    e->cfg = *cfg;
    e->cfg.max_batch_tokens = std::min(std::max(cfg->max_batch_tokens, 64), cfg->cap_tokens);  // src/main.rs:153
    e->st = stream;
    e->cap_markers = cfg->cap_tokens / 2 + 64;  // src/model.rs:278
    e->n_attn = d1h_model_layers(m, 1);
    e->n_conv = d1h_model_layers(m, 0);
    e->vision_patches = vision ? d1h_vision_capacity(vision) : 0;
    cudaGetDevice(&e->device);
    // media prefixes and their embeddings are stream-ordered allocations from the device's default pool; keep
    // freed blocks in the pool instead of unmapping them at every synchronisation (a process-local setting)
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, e->device) == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    e->ws = d1h_workspace_create(m, cfg->cap_tokens);
    if (!e->ws) {
        efail(std::string("workspace: ") + d1h_last_error());
        delete e;
        return nullptr;
    }
    e->logit_buf.resize(e->cap_markers + 16);
    return e;
}

void d1e_destroy(D1Engine* e) {
    if (!e) return;
    cudaSetDevice(e->device);
    while (!e->inflight.empty()) {
        InFlight f = e->inflight.front();
        e->inflight.pop_front();
        e->complete(f);
    }
    for (auto& [id, js] : e->jobs)
        if (js.has_prefix) d1h_prefix_free(&js.prefix, e->st);
    cudaStreamSynchronize(e->st);
    d1h_workspace_destroy(e->ws);
    delete e;
}

long long d1e_submit(D1Engine* e, const D1Job* job) {
    if (!e || !job || job->n_rows < 0 || (job->n_rows > 0 && !job->rows)) return efail("bad job");
    JobState js;
    js.id = e->next_id++;
    for (int i = 0; i < job->n_rows; i++) {
        const D1Row& r = job->rows[i];
        if (r.n_ids < 0 || r.n_markers < 0 || (r.n_ids && !r.ids) || (r.n_markers && !r.markers)) return efail("bad row");
        Row row;
        row.ids.assign(r.ids, r.ids + r.n_ids);
        row.markers.assign(r.markers, r.markers + r.n_markers);
        for (int mk : row.markers)
            if (mk < 0 || mk >= r.n_ids) return efail("marker outside its row");
        row.qtype = r.qtype;
        js.rows.push_back(std::move(row));
    }
    js.results.resize(js.rows.size());
    const D1Media& md = job->media;
    js.kind = md.kind;
    if (md.kind == D1_MEDIA_IMAGES) {
        if (md.n_crops <= 0 || !md.ph || !md.pw || !md.patches) return efail("bad image media");
        size_t np = 0;
        for (int i = 0; i < md.n_crops; i++) {
            if (md.ph[i] <= 0 || md.pw[i] <= 0 || (md.ph[i] & 1) || (md.pw[i] & 1)) return efail("bad crop grid");
            np += (size_t)md.ph[i] * md.pw[i];
        }
        js.ph.assign(md.ph, md.ph + md.n_crops);
        js.pw.assign(md.pw, md.pw + md.n_crops);
        const uint16_t* p = reinterpret_cast<const uint16_t*>(md.patches);
        js.patches.assign(p, p + np * 768);
    } else if (md.kind == D1_MEDIA_AUDIO) {
        if (md.pcm) {
            const int rate = md.sample_rate ? md.sample_rate : 16000;
            if (md.n_samples < 0 || rate <= 0) return efail("bad audio media");
            // 16 kHz: cut to 30 s (src/audio.rs:241-247); another rate: what the WAV decoder keeps (30 s + 1 s,
            // :59), resampled on the device, then cut to 30 s
            const int n = rate == 16000 ? std::min(md.n_samples, 30 * 16000)
                                        : (int)std::min<long long>(md.n_samples, 31ll * rate);
            const int n16 = rate == 16000 ? n : d1_resample_len(n, rate, 16000);
            if (n16 < 0) return efail("bad audio sample rate");
            js.pcm.assign(md.pcm, md.pcm + n);
            js.rate = rate;
            js.valid = std::max(std::min(n16, 30 * 16000), 8000) / 160;
        } else {
            if (md.valid < 1 || md.valid > 3000 || !md.mel) return efail("bad audio media");
            js.valid = md.valid;
            js.mel.assign(md.mel, md.mel + (size_t)md.valid * 128);
        }
    } else if (md.kind != D1_MEDIA_NONE) {
        return efail("unknown media kind");
    }
    js.media_done = md.kind == D1_MEDIA_NONE;
    const long long id = js.id;
    if (js.rows.empty() && js.media_done) {  // nothing to run
        e->done.push_back(Done{id, {}, ""});
        return id;
    }
    e->jobs.emplace(id, std::move(js));
    e->order.push_back(id);
    return id;
}

int d1e_step(D1Engine* e) {
    if (!e) return efail("null engine");
    cudaSetDevice(e->device);
    return e->step();
}

int d1e_pending(const D1Engine* e) { return e ? (int)e->jobs.size() : 0; }

long long d1e_queued_tokens(const D1Engine* e) {
    if (!e) return 0;
    long long t = 0;
    for (const auto& [id, js] : e->jobs) {
        for (size_t r = js.next_row; r < js.rows.size(); r++) t += (long long)js.rows[r].ids.size();
        if (!js.media_done) t += (long long)js.prefix_len();
    }
    return t;
}

int d1e_take(D1Engine* e, long long* id, float* logits, int cap, char* err, int err_cap) {
    if (!e || !id || e->done.empty()) return -1;
    Done& d = e->done.front();
    const int n = (int)d.logits.size();
    if (n > cap) return efail("logit buffer too small (need " + std::to_string(n) + ")", -2);
    *id = d.id;
    if (n) memcpy(logits, d.logits.data(), (size_t)n * 4);
    if (err && err_cap > 0) {
        strncpy(err, d.err.c_str(), (size_t)err_cap - 1);
        err[err_cap - 1] = 0;
    }
    e->done.pop_front();
    return n;
}

int d1e_next_logits(const D1Engine* e) { return e && !e->done.empty() ? (int)e->done.front().logits.size() : -1; }

void d1e_stats(const D1Engine* e, D1EngineStats* s) {
    if (!e || !s) return;
    s->tokens = e->st_tokens;
    s->media_tokens = e->st_media_tokens;
    s->batches = e->st_batches;
    s->media_jobs = e->st_media;
    s->rows = e->st_rows;
}

const char* d1e_last_error(void) { return e_err.c_str(); }

}  // extern "C"
