/* st_loader.cu: open one layer's MoE block from an MLX checkpoint directory (*.safetensors shards).
 *
 * The reference reads its checkpoints with a safetensors reader of its own (engine/src/io/k3_st.c:509-633:
 * every *.safetensors file of a directory, one flat JSON header per shard) and builds the block in load_moe
 * (engine/src/model.c:52-70): tensors <prefix>.switch_mlp.{gate,up,down}_proj, <prefix>.gate (router),
 * <prefix>.shared_expert.{gate,up,down}_proj and <prefix>.shared_expert_gate, each as .weight (U32 packed
 * codes), .scales and .biases (BF16), in the MLX affine layout (engine/include/qmat.h:3-11). Shapes follow
 * loader.c:16-41: cols = groups * group_size, bits = packed * 32 / cols; the routed experts are [E][rows][...].
 *
 * Here the shards are memory-mapped, the tensors are checked (dtype, shape, bounds) and handed to
 * qe_moe_create, which copies them (or this rank's expert slice) into HBM; the mappings are released before
 * returning. Host code only.
 */
#include "ckpt.h"

using namespace qe_ckpt;

extern "C" {

int qe_safetensors_tensor_info(const char *dir, const char *name, char *dtype, int64_t *shape, int *ndim) {
    if (!dir || !name || !dtype || !shape || !ndim) QE_FAIL("safetensors: bad arguments");
    Checkpoint ck;
    if (ck.open_dir(dir)) return -1;
    const TensorInfo *t = ck.find(name);
    if (!t) QE_FAIL("safetensors: no tensor %s in %s", name, dir);
    if (t->shape.size() > 8) QE_FAIL("safetensors: %s has rank %zu > 8", name, t->shape.size());
    snprintf(dtype, 8, "%s", t->dtype.c_str());
    for (size_t i = 0; i < t->shape.size(); i++) shape[i] = t->shape[i];
    *ndim = (int)t->shape.size();
    return 0;
}

QeMoe *qe_moe_open_safetensors(const char *dir, const char *prefix, const QeMoeConfig *cfg_in) {
    if (!dir || !prefix || !cfg_in) {
        fprintf(stderr, "qengine_b200: open_safetensors: bad arguments\n");
        return nullptr;
    }
    Checkpoint ck;
    if (ck.open_dir(dir)) return nullptr;
    const std::string p = prefix;
    QView gate, up, down, sg, su, sd, rq, srq;
    if (qview(ck, p + ".switch_mlp.gate_proj", 3, gate) || qview(ck, p + ".switch_mlp.up_proj", 3, up) ||
        qview(ck, p + ".switch_mlp.down_proj", 3, down) || qview(ck, p + ".shared_expert.gate_proj", 2, sg) ||
        qview(ck, p + ".shared_expert.up_proj", 2, su) || qview(ck, p + ".shared_expert.down_proj", 2, sd) ||
        qview(ck, p + ".gate", 2, rq) || qview(ck, p + ".shared_expert_gate", 2, srq))
        return nullptr;
    QeMoeConfig c = *cfg_in;
    const int gs = c.group_size;
    if (gs != 32 && gs != 64 && gs != 128) {
        fprintf(stderr, "qengine_b200: open_safetensors: group_size %d not in {32, 64, 128}\n", gs);
        return nullptr;
    }
    /* shapes as loader.c:26 derives them: cols = groups * gs, bits = packed * 32 / cols */
    const int64_t hidden = gate.groups * gs, inter = down.groups * gs, sh_inter = sd.groups * gs;
    const int64_t bits = hidden ? gate.packed * 32 / hidden : 0, rbits = hidden ? rq.packed * 32 / hidden : 0;
    const bool shapes_ok =
        hidden > 0 && (bits == 4 || bits == 8) && gate.packed * 32 == bits * hidden && up.n == gate.n &&
        down.n == gate.n && up.rows == gate.rows && up.packed == gate.packed && gate.rows == inter &&
        down.rows == hidden && down.packed * 32 == bits * inter && sg.rows == sh_inter && su.rows == sh_inter &&
        sg.packed == gate.packed && su.packed == gate.packed && sd.rows == hidden && sd.packed * 32 == bits * sh_inter &&
        rq.rows == gate.n && (rbits == 4 || rbits == 8) && rq.packed * 32 == rbits * hidden && srq.rows == 1 &&
        srq.packed == rq.packed;
    if (!shapes_ok) {
        fprintf(stderr, "qengine_b200: open_safetensors: %s: tensor shapes do not form one MoE block\n", prefix);
        return nullptr;
    }
    auto check = [&](int given, int64_t found, const char *what) {
        if (given && given != found) {
            fprintf(stderr, "qengine_b200: open_safetensors: %s=%d given, checkpoint has %lld\n", what, given,
                    (long long)found);
            return false;
        }
        return true;
    };
    if (!check(c.hidden, hidden, "hidden") || !check(c.E, gate.n, "E") || !check(c.inter, inter, "inter") ||
        !check(c.sh_inter, sh_inter, "sh_inter") || !check(c.bits, bits, "bits"))
        return nullptr;
    c.hidden = (int)hidden;
    c.E = (int)gate.n;
    c.inter = (int)inter;
    c.sh_inter = (int)sh_inter;
    c.bits = (int)bits;
    c.router_mode = QE_ROUTER_QMAT;
    c.router_bits = (int)rbits;
    QeMoeWeights w = {};
    w.router_q = rq.t;
    w.sh_router_q = srq.t;
    w.gate = gate.t;
    w.up = up.t;
    w.down = down.t;
    w.sh_gate = sg.t;
    w.sh_up = su.t;
    w.sh_down = sd.t;
    return qe_moe_create(&c, &w);   /* copies into HBM; the mappings go away with ck */
}

}  // extern "C"
