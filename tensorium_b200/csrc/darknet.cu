// darknet.cu -- darknet .cfg / .weights files for the whole-network executor: the B200 build's
// TDarknetParser (source/nparser.pas) and TCFGList (source/nconfig.pas).
//
// Host code only. The loader builds the network through the public tb_net_add_* calls, reading
// each layer's arrays from the .weights stream right after the layer's shape is known, so the
// file is read once, front to back. Connected-layer batchnorm is folded on load (the executor's
// fully connected kernel has no separate batchnorm pass); conv batchnorm stays unfolded so that
// tb_net_fuse_batchnorm (TNNet.fuseBatchNorm) decides, as for a net built layer by layer.
#include "common.cuh"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace tbi;

namespace {

// ---- .cfg text (TCFGList.loadFromFile, source/nconfig.pas:280-323) -----------------------------

struct Section {
    std::string type;                  // lower-cased section name
    std::vector<std::string> options;  // "key=value" lines, file order
    int line = 0;                      // line of the section header (for messages)
};

// stripChars (source/nconfig.pas:60-69): drop blanks and tabs from every position but the last
// (its loop stops one short of the end; the trailing character is trimmed later anyway).
std::string strip_blanks(const std::string& s) {
    std::string r;
    for (size_t j = 0; j < s.size(); ++j)
        if (j + 1 == s.size() || (s[j] != ' ' && s[j] != '\t')) r.push_back(s[j]);
    return r;
}

// stripComments (source/nconfig.pas:71-82): cut at the first ';' or '#'.
std::string strip_comment(const std::string& s) {
    size_t p = s.find_first_of(";#");
    return p == std::string::npos ? s : s.substr(0, p);
}

std::string trim(const std::string& s) {
    size_t a = 0, b = s.size();
    while (a < b && (unsigned char)s[a] <= ' ') ++a;
    while (b > a && (unsigned char)s[b - 1] <= ' ') --b;
    return s.substr(a, b - a);
}

std::string lower(std::string s) {
    for (char& ch : s) if (ch >= 'A' && ch <= 'Z') ch = (char)(ch - 'A' + 'a');
    return s;
}

int read_cfg(const char* path, std::vector<Section>& out) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return fail(TB_ERR_INVALID, "cfg file %s: %s", path, std::strerror(errno));
    std::string text;
    char buf[65536];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, got);
    std::fclose(f);
    int lineno = 0;
    size_t pos = 0;
    while (pos < text.size()) {
        size_t e = text.find('\n', pos);
        if (e == std::string::npos) e = text.size();
        std::string line = text.substr(pos, e - pos);
        pos = e + 1;
        ++lineno;
        if (!line.empty() && line.back() == '\r') line.pop_back();
        line = strip_comment(strip_blanks(line));
        line = trim(line);
        if (line.empty()) continue;
        if (line[0] == '[') {
            Section s;
            std::string name = line.substr(1);
            if (!name.empty() && name.back() == ']') name.pop_back();
            s.type = lower(name);
            s.line = lineno;
            out.push_back(std::move(s));
        } else {
            if (out.empty())
                return fail(TB_ERR_INVALID, "cfg line %d: option before the first section", lineno);
            // TCFGSection.addOptionLine (source/nconfig.pas:162-174): lines without '=' are
            // reported and skipped
            if (line.find('=') != std::string::npos) out.back().options.push_back(line);
        }
    }
    return TB_OK;
}

// TCFGSection lookups (source/nconfig.pas:176-258): the first "key=" line wins.
struct Opts {
    const Section& s;
    int index;      // layer index (-1 for [net]) for messages
    int err = TB_OK;

    bool find(const char* key, std::string& val) const {
        for (const std::string& o : s.options) {
            size_t p = o.find('=');
            if (trim(o.substr(0, p)) == key) { val = trim(o.substr(p + 1)); return true; }
        }
        return false;
    }
    bool has(const char* key) const { std::string v; return find(key, v); }
    int64_t i(const char* key, int64_t def) {
        std::string v;
        if (!find(key, v)) return def;
        char* end = nullptr;
        errno = 0;
        long long x = std::strtoll(v.c_str(), &end, 10);
        if (v.empty() || *end || errno) {
            if (err == TB_OK) err = fail(TB_ERR_INVALID, "cfg [%s] line %d: %s=%s is not an integer",
                                         s.type.c_str(), s.line, key, v.c_str());
            return def;
        }
        return (int64_t)x;
    }
    float f(const char* key, float def) {
        std::string v;
        if (!find(key, v)) return def;
        char* end = nullptr;
        float x = std::strtof(v.c_str(), &end);
        if (v.empty() || *end) {
            if (err == TB_OK) err = fail(TB_ERR_INVALID, "cfg [%s] line %d: %s=%s is not a number",
                                         s.type.c_str(), s.line, key, v.c_str());
            return def;
        }
        return x;
    }
    bool b(const char* key, bool def) { return i(key, def ? 1 : 0) != 0; }
    std::string str(const char* key, const char* def) const {
        std::string v;
        return find(key, v) ? v : std::string(def);
    }
};

std::vector<std::string> split_commas(const std::string& s) {
    std::vector<std::string> r;
    size_t a = 0;
    while (true) {
        size_t e = s.find(',', a);
        r.push_back(trim(s.substr(a, e == std::string::npos ? std::string::npos : e - a)));
        if (e == std::string::npos) break;
        a = e + 1;
    }
    return r;
}

// TActivationTypeHelper.fromString (source/nparser.pas:1584-1611); unknown names give relu, as
// there. Names the executor has no kernel for (swish, mish, gelu, ...) are reported by the
// layer's add call.
int64_t activation_of(std::string s) {
    s = lower(s);
    static const struct { const char* name; int64_t act; } table[] = {
        {"logistic", TB_ACT_LOGISTIC}, {"loggy", TB_ACT_LOGGY}, {"relu", TB_ACT_RELU},
        {"relu6", TB_ACT_RELU6}, {"elu", TB_ACT_ELU}, {"selu", TB_ACT_SELU}, {"relie", TB_ACT_RELIE},
        {"plse", TB_ACT_PLSE}, {"hardtan", TB_ACT_HARDTAN}, {"lhtan", TB_ACT_LHTAN},
        {"linear", TB_ACT_LINEAR}, {"ramp", TB_ACT_RAMP}, {"revleaky", TB_ACT_REVLEAKY},
        {"leaky", TB_ACT_LEAKY}, {"tanh", TB_ACT_TANH},
    };
    for (const auto& t : table) if (s == t.name) return t.act;
    static const char* other[] = {"swish", "mish", "hard_mish", "normalize_channels",
                                  "normalize_channels_softmax", "normalize_channels_softmax_maxval",
                                  "gelu", "stair"};
    for (const char* o : other) if (s == o) return -1;  // a reference activation without a kernel here
    return TB_ACT_RELU;
}

// ---- .weights stream (TDarknetParser.loadWeights, source/nparser.pas:1275-1340) ---------------

struct WeightsIn {
    FILE* f = nullptr;
    bool transpose = false;
    bool at_eof = false;    // the reference stops reading at the first layer boundary at EOF
    ~WeightsIn() { if (f) std::fclose(f); }

    int open(const char* path) {
        f = std::fopen(path, "rb");
        if (!f) return fail(TB_ERR_INVALID, "weights file %s: %s", path, std::strerror(errno));
        int32_t hdr[3];
        if (std::fread(hdr, 4, 3, f) != 3) return fail(TB_ERR_INVALID, "weights file %s: short header", path);
        const int64_t major = (uint32_t)hdr[0], minor = (uint32_t)hdr[1];
        // seen is 64-bit from version 0.2 on (major * 10 + minor >= 2), 32-bit before
        const size_t seen_bytes = major * 10 + minor >= 2 ? 8 : 4;
        unsigned char seen[8];
        if (std::fread(seen, 1, seen_bytes, f) != seen_bytes)
            return fail(TB_ERR_INVALID, "weights file %s: short header", path);
        transpose = major > 1000 || minor > 1000;
        check_eof();
        return TB_OK;
    }
    void check_eof() {
        int ch = std::fgetc(f);
        if (ch == EOF) at_eof = true;
        else std::ungetc(ch, f);
    }
    int read(std::vector<float>& v, int layer, const char* what) {
        if (v.empty()) return TB_OK;
        size_t got = std::fread(v.data(), sizeof(float), v.size(), f);
        if (got != v.size())
            return fail(TB_ERR_INVALID, "weights file ends inside layer %d (%s: %zu of %zu floats)",
                        layer, what, got, v.size());
        return TB_OK;
    }
};

struct Builder {
    tb_net* net = nullptr;
    WeightsIn* win = nullptr;   // null: no weights file
    int64_t cutoff = 0;

    int last_shape(int64_t* c, int64_t* h, int64_t* w) {
        int64_t n = 0;
        tb_net_layer_count(net, &n);
        if (n == 0) return tb_net_input_shape(net, nullptr, c, h, w);
        tb_layer_info d;
        int r = tb_net_layer_info(net, n - 1, &d);
        if (r != TB_OK) return r;
        *c = d.out_c; *h = d.out_h; *w = d.out_w;
        return TB_OK;
    }
    bool reads(int index) const {
        return win && !win->at_eof && (cutoff <= 0 || index < cutoff);
    }
};

int unsupported(const Section& s, const char* what) {
    return fail(TB_ERR_UNSUPPORTED, "cfg [%s] line %d: %s", s.type.c_str(), s.line, what);
}

// parseConvolutional (source/nparser.pas:154-246) + loadConvolutionalWeights (:1140-1210)
int add_conv(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const int64_t filters = o.i("filters", 1);
    const int64_t groups = o.i("groups", 1);
    const int64_t size = o.i("size", 1);
    int64_t stride_x = o.i("stride_x", -1), stride_y = o.i("stride_y", -1);
    if (stride_x < 1 || stride_y < 1) {
        const int64_t stride = o.i("stride", 1);
        if (stride_x < 1) stride_x = stride;
        if (stride_y < 1) stride_y = stride;
    }
    int64_t dilation = o.i("dilation", 1);
    if (size == 1) dilation = 1;
    int64_t padding = o.i("padding", 0);
    if (o.b("pad", false)) padding = size / 2;
    const int64_t act = activation_of(o.str("activation", "logistic"));
    int64_t bn = o.i("batch_normalize", 0);
    if (o.b("cbn", false)) bn = 2;
    if (o.err) return o.err;
    if (groups != 1) return unsupported(s, "grouped convolution (groups != 1)");
    if (stride_x != stride_y) return unsupported(s, "stride_x != stride_y");
    if (dilation != 1) return unsupported(s, "dilation != 1");
    if (o.i("antialiasing", 0) != 0) return unsupported(s, "antialiasing");
    if (o.has("share_index")) return unsupported(s, "share_index");
    if (o.i("sway", 0) || o.i("rotate", 0) || o.i("stretch", 0) || o.i("stretch_sway", 0))
        return unsupported(s, "deformable (sway / rotate / stretch) convolution");
    if (o.i("assisted_excitation", 0) != 0) return unsupported(s, "assisted_excitation");
    if (act < 0) return unsupported(s, "activation without a kernel in this build");
    int64_t c, h, w;
    int r = B.last_shape(&c, &h, &w);
    if (r != TB_OK) return r;
    if (h * w * c == 0) return unsupported(s, "the layer before a convolution must output an image");
    const bool batchnorm = bn == 1 || bn == 2;
    std::vector<float> wt((size_t)(filters * c * size * size), 0.0f), bias((size_t)filters, 0.0f);
    std::vector<float> scales((size_t)filters, 1.0f), mean((size_t)filters, 0.0f), var((size_t)filters, 1.0f);
    if (B.reads(index) && !o.b("dontload", false)) {
        if ((r = B.win->read(bias, index, "biases")) != TB_OK) return r;
        if (batchnorm && !o.b("dontloadscales", false)) {
            if ((r = B.win->read(scales, index, "scales")) != TB_OK) return r;
            if ((r = B.win->read(mean, index, "rolling_mean")) != TB_OK) return r;
            if ((r = B.win->read(var, index, "rolling_variance")) != TB_OK) return r;
        }
        if ((r = B.win->read(wt, index, "weights")) != TB_OK) return r;
        B.win->check_eof();
    }
    return tb_net_add_conv(B.net, filters, size, stride_x, padding, act, batchnorm ? 1 : 0, wt.data(),
                           bias.data(), scales.data(), mean.data(), var.data());
}

// parseConnected (source/nparser.pas:146-152) + loadConnectedWeights (:1102-1128)
int add_connected(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const int64_t outputs = o.i("output", 1);
    const int64_t act = activation_of(o.str("activation", "relu"));
    const bool batchnorm = o.b("batch_normalize", false);
    if (o.err) return o.err;
    if (act < 0) return unsupported(s, "activation without a kernel in this build");
    int64_t c, h, w;
    int r = B.last_shape(&c, &h, &w);
    if (r != TB_OK) return r;
    const int64_t inputs = c * h * w;
    std::vector<float> wt((size_t)(outputs * inputs), 0.0f), bias((size_t)outputs, 0.0f);
    if (B.reads(index) && !o.b("dontload", false)) {
        if ((r = B.win->read(bias, index, "biases")) != TB_OK) return r;
        if ((r = B.win->read(wt, index, "weights")) != TB_OK) return r;
        if (B.win->transpose) {  // stored [inputs][outputs]
            std::vector<float> t(wt.size());
            for (int64_t i = 0; i < inputs; ++i)
                for (int64_t j = 0; j < outputs; ++j) t[(size_t)(j * inputs + i)] = wt[(size_t)(i * outputs + j)];
            wt.swap(t);
        }
        if (batchnorm && !o.b("dontloadscales", false)) {
            std::vector<float> scales((size_t)outputs), mean((size_t)outputs), var((size_t)outputs);
            if ((r = B.win->read(scales, index, "scales")) != TB_OK) return r;
            if ((r = B.win->read(mean, index, "rolling_mean")) != TB_OK) return r;
            if ((r = B.win->read(var, index, "rolling_variance")) != TB_OK) return r;
            r = tb_conv_fold_bn(outputs, inputs, wt.data(), bias.data(), scales.data(), mean.data(), var.data());
            if (r != TB_OK) return r;
        }
        B.win->check_eof();
    }
    return tb_net_add_connected(B.net, outputs, act, wt.data(), bias.data());
}

// parseMaxPool (source/nparser.pas:248-269)
int add_maxpool(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const int64_t stride = o.i("stride", 1);
    const int64_t stride_x = o.i("stride_x", stride), stride_y = o.i("stride_y", stride);
    const int64_t size = o.i("size", stride);
    const int64_t padding = o.i("padding", size - 1);
    if (o.err) return o.err;
    if (stride_x != stride_y) return unsupported(s, "stride_x != stride_y");
    if (o.i("maxpool_depth", 0) != 0) return unsupported(s, "maxpool_depth");
    if (o.i("antialiasing", 0) != 0) return unsupported(s, "antialiasing");
    return tb_net_add_maxpool(B.net, size, stride_x, padding);
}

// parseConcat (source/nparser.pas:333-403): negative indices are relative to this layer
int add_route(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const std::string l = o.str("layers", "");
    if (l.empty()) return unsupported(s, "route layer must specify input layers");
    if (o.i("groups", 1) != 1) return unsupported(s, "route groups != 1");
    if (o.err) return o.err;
    std::vector<int64_t> layers;
    for (const std::string& v : split_commas(l)) {
        char* end = nullptr;
        long long x = std::strtoll(v.c_str(), &end, 10);
        if (v.empty() || *end) return fail(TB_ERR_INVALID, "cfg [route] line %d: bad layer %s", s.line, v.c_str());
        layers.push_back(x < 0 ? index + x : x);
    }
    return tb_net_add_route(B.net, (int64_t)layers.size(), layers.data());
}

// parseAdd (source/nparser.pas:405-487)
int add_shortcut(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const int64_t act = activation_of(o.str("activation", "linear"));
    const std::string wt = o.str("weights_type", "none");
    const std::string from = o.str("from", "");
    if (o.err) return o.err;
    if (from.empty()) return unsupported(s, "shortcut must specify input layers: from = ...");
    if (wt != "none") return unsupported(s, "weighted shortcut (weights_type)");
    if (act < 0) return unsupported(s, "activation without a kernel in this build");
    std::vector<std::string> v = split_commas(from);
    if (v.size() != 1) return unsupported(s, "shortcut from more than one layer");
    char* end = nullptr;
    long long x = std::strtoll(v[0].c_str(), &end, 10);
    if (v[0].empty() || *end) return fail(TB_ERR_INVALID, "cfg [shortcut] line %d: bad from=%s", s.line, v[0].c_str());
    return tb_net_add_shortcut(B.net, x < 0 ? index + x : x, act);
}

// parseYolo (source/nparser.pas:516-644) and TYoloLayer.Create's defaults
// (source/nyololayer.pas:301-327: mask 0..n-1, anchors 0.5)
int add_yolo(Builder& B, const Section& s, int index) {
    Opts o{s, index};
    const int64_t classes = o.i("classes", 20);
    const int64_t total = o.i("num", 1);
    const float scale_xy = o.f("scale_x_y", 1.0f);
    const bool new_coords = o.b("new_coords", false);
    if (o.err) return o.err;
    if (new_coords) return unsupported(s, "new_coords");
    if (total <= 0) return unsupported(s, "num must be positive");
    std::vector<int64_t> mask;
    const std::string m = o.str("mask", "");
    if (m.empty()) {
        for (int64_t k = 0; k < total; ++k) mask.push_back(k);
    } else {
        for (const std::string& v : split_commas(m)) {
            char* end = nullptr;
            long long x = std::strtoll(v.c_str(), &end, 10);
            if (v.empty() || *end) return fail(TB_ERR_INVALID, "cfg [yolo] line %d: bad mask %s", s.line, v.c_str());
            mask.push_back(x);
        }
    }
    std::vector<float> anchors((size_t)(2 * total), 0.5f);
    const std::string a = o.str("anchors", "");
    if (!a.empty()) {
        std::vector<std::string> v = split_commas(a);
        for (size_t k = 0; k < v.size() && k < anchors.size(); ++k) {
            char* end = nullptr;
            float x = std::strtof(v[k].c_str(), &end);
            if (v[k].empty() || *end) return fail(TB_ERR_INVALID, "cfg [yolo] line %d: bad anchor %s", s.line, v[k].c_str());
            anchors[k] = x;
        }
    }
    return tb_net_add_yolo(B.net, classes, (int64_t)mask.size(), mask.data(), total, anchors.data(), scale_xy);
}

int add_section(Builder& B, const Section& s, int index) {
    const std::string& t = s.type;
    if (t == "convolutional" || t == "conv") return add_conv(B, s, index);
    if (t == "connected" || t == "conn") return add_connected(B, s, index);
    if (t == "maxpool" || t == "max") return add_maxpool(B, s, index);
    if (t == "avgpool" || t == "avg") return tb_net_add_avgpool(B.net);
    if (t == "route") return add_route(B, s, index);
    if (t == "shortcut") return add_shortcut(B, s, index);
    if (t == "upsample") {  // parseUpSample (source/nparser.pas:506-509)
        Opts o{s, index};
        const int64_t stride = o.i("stride", 2);
        const float scale = o.f("scale", 1.0f);
        if (o.err) return o.err;
        if (stride <= 0) return unsupported(s, "downsampling (negative stride) upsample");
        return tb_net_add_upsample(B.net, stride, scale);
    }
    if (t == "yolo") return add_yolo(B, s, index);
    if (t == "softmax" || t == "soft") {  // parseSoftmax (source/nparser.pas:722-738)
        Opts o{s, index};
        const int64_t groups = o.i("groups", 1);
        const float temperature = o.f("temperature", 1.0f);
        if (o.err) return o.err;
        if (!o.str("tree", "").empty()) return unsupported(s, "hierarchical softmax (tree)");
        return tb_net_add_softmax(B.net, groups, temperature);
    }
    if (t == "dropout") {
        // TDropoutLayer.forward (source/ndropoutlayer.pas:82-110) passes its input through when
        // not training: a one-input route keeps the cfg's layer numbering
        const int64_t prev = index - 1;
        if (prev < 0) return unsupported(s, "dropout as the first layer");
        return tb_net_add_route(B.net, 1, &prev);
    }
    return unsupported(s, "layer type not in the inference executor");
}

}  // namespace

extern "C" {

int tb_darknet_load(tb_ctx* ctx, const char* cfg_path, const char* weights_path, int64_t batch,
                    int64_t cutoff, tb_net** out) {
    if (!cfg_path || !out) return fail(TB_ERR_INVALID, "tb_darknet_load: null argument");
    *out = nullptr;
    std::vector<Section> secs;
    int r = read_cfg(cfg_path, secs);
    if (r != TB_OK) return r;
    if (secs.empty() || (secs[0].type != "net" && secs[0].type != "network"))
        return fail(TB_ERR_INVALID, "cfg %s: the first section must be [net]", cfg_path);
    // parseNet (source/nparser.pas:942-1000) + TDarknetParser.Create's batch override (:800-801)
    Opts n{secs[0], -1};
    const int64_t mini = n.i("batch", 1), subdivs = n.i("subdivisions", 1), steps = n.i("time_steps", 1);
    const int64_t h = n.i("height", 0), w = n.i("width", 0), c = n.i("channels", 0);
    const int64_t inputs = n.i("inputs", 0);
    if (n.err) return n.err;
    if (subdivs <= 0 || mini < subdivs || mini % subdivs)
        return fail(TB_ERR_INVALID, "cfg [net]: batch must be a multiple of subdivisions");
    int64_t nb = mini / subdivs * steps;
    if (batch > 0 && nb * subdivs != batch) nb = batch;
    int64_t ic = c, ih = h, iw = w;
    if (h * w * c == 0) { ic = inputs; ih = 1; iw = 1; }
    if (ic <= 0) return fail(TB_ERR_INVALID, "cfg [net]: no input shape (height/width/channels or inputs)");
    tb_net* net = nullptr;
    r = tb_net_create(ctx, nb, ic, ih, iw, &net);
    if (r != TB_OK) return r;
    WeightsIn win;
    Builder B;
    B.net = net;
    B.cutoff = cutoff;
    if (weights_path) {
        r = win.open(weights_path);
        if (r != TB_OK) { tb_net_destroy(net); return r; }
        B.win = &win;
    }
    for (size_t k = 1; k < secs.size(); ++k) {
        r = add_section(B, secs[k], (int)(k - 1));
        if (r < 0) { tb_net_destroy(net); return r; }
    }
    *out = net;
    return TB_OK;
}

int tb_darknet_save_weights(tb_net* net, const char* weights_path, int64_t seen) {
    if (!net || !weights_path) return fail(TB_ERR_INVALID, "tb_darknet_save_weights: null argument");
    int64_t n = 0;
    int r = tb_net_layer_count(net, &n);
    if (r != TB_OK) return r;
    std::vector<std::vector<float>> blocks;
    for (int64_t i = 0; i < n; ++i) {
        tb_layer_info d;
        if ((r = tb_net_layer_info(net, i, &d)) != TB_OK) return r;
        if (d.type != TB_LAYER_CONV && d.type != TB_LAYER_CONNECTED) continue;
        std::vector<int64_t> order = {TB_PARAM_BIASES};
        if (d.type == TB_LAYER_CONV && d.batch_normalize)
            order.insert(order.end(), {TB_PARAM_SCALES, TB_PARAM_ROLLING_MEAN, TB_PARAM_ROLLING_VAR});
        order.push_back(TB_PARAM_WEIGHTS);
        for (int64_t which : order) {
            int64_t cnt = 0;
            if ((r = tb_net_layer_param(net, i, which, nullptr, 0, &cnt)) != TB_OK) return r;
            std::vector<float> v((size_t)cnt);
            if ((r = tb_net_layer_param(net, i, which, v.data(), cnt, nullptr)) != TB_OK) return r;
            blocks.push_back(std::move(v));
        }
    }
    FILE* f = std::fopen(weights_path, "wb");
    if (!f) return fail(TB_ERR_INVALID, "weights file %s: %s", weights_path, std::strerror(errno));
    const int32_t hdr[3] = {0, 2, 5};
    const uint64_t s64 = (uint64_t)seen;
    bool ok = std::fwrite(hdr, 4, 3, f) == 3 && std::fwrite(&s64, 8, 1, f) == 1;
    for (const auto& v : blocks)
        ok = ok && (v.empty() || std::fwrite(v.data(), sizeof(float), v.size(), f) == v.size());
    ok = (std::fclose(f) == 0) && ok;
    if (!ok) return fail(TB_ERR_INVALID, "weights file %s: write failed", weights_path);
    return TB_OK;
}

}  // extern "C"
