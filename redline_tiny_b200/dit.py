"""The DiT denoise step on B200, composed from the hot-path kernels (config 4).

Follows the reference's block sequence (redline/forward.py:240-254, CachedStep.blocks; step structure
forward.py:396-412, 256-269, 605):

    per block i:  qkv = a @ Wqkv_i -> qkv_post (QK-RMSNorm * w, RoPE) -> attention -> c = o @ Wo_i
                  x1, a2 = ln_mod(x0, c, p_mlp)          (x1 = x0 + tanh(g1) c; a2 = LN(x1) (1 + s2))
                  h = SwiGLU(a2 @ Wup_i) -> c = h @ Wdown_i
                  x0, a = ln_mod(x1, c, p_attn | p_out)  (x0 = x1 + tanh(g2) c; a = LN(x0) (1 + s1 | out scale))
    per step:     x = [text rows | img_in(latents)], a = LN1 -> 32 blocks -> proj_out on the image rows ->
                  Euler step on the host.

The adaLN modulation is shared by all blocks ([scale1 | gate1 | scale2 | gate2], host_glue.modulation), with two
parameter rows: rows below `row_split` (the text prefix) use the t = 0 row, as the reference's ln_mod S split does.
All activations stay on the GPU in bf16 row-major; every linear is the packed-weight bfp16 GEMM.
"""

import math

import numpy as np
import torch

from . import host_glue as HG
from . import ops
from . import _lib as L

HEAD_DIM = 128
C_LOG2 = math.log2(math.e) / math.sqrt(HEAD_DIM)   # folded into w_q as the reference does (forward.py:226-228)


class DiTConfig:
    def __init__(self, hidden=3072, heads=24, ffn=12288, blocks=32, text=256, image=4096, latent_ch=64,
                 temb_dim=256, grid=(64, 64)):
        assert hidden == heads * HEAD_DIM and grid[0] * grid[1] == image
        self.hidden, self.heads, self.ffn, self.blocks = hidden, heads, ffn, blocks
        self.text, self.image, self.latent_ch, self.temb_dim, self.grid = text, image, latent_ch, temb_dim, grid
        self.M = text + image

    def flop_per_step(self):
        M, D, F = self.M, self.hidden, self.ffn
        per_block = 2 * M * D * 3 * D + 2 * M * D * D + 2 * M * D * 2 * F + 2 * M * F * D + 4 * self.heads * M * M * 128
        return self.blocks * per_block + 2 * self.image * self.latent_ch * D + 2 * self.image * D * 128


def random_weights(cfg, seed=0, device="cuda"):
    """Random-init weights of the config's architecture (there is no checkpoint): linears N(0, 0.02) as float
    B = W^T (K, N); QK-norm weights N(1, 0.1); small host weights for the timestep embedding and modulation.
    Drawn on `device` from a seeded generator (config 4 has 4.8 G weights)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    D, F = cfg.hidden, cfg.ffn

    def randn(*shape, std=0.02):
        return (torch.randn(*shape, generator=g, device=device) * std).float()

    blocks = []
    for _ in range(cfg.blocks):
        blocks.append({
            "qkv": randn(D, 3 * D), "o": randn(D, D),
            "gate": randn(F, D), "proj": randn(F, D),           # W (out F, in D), as interleave_up takes them
            "down": randn(F, D),                                  # B = W_down^T (K = F, N = D)
            "norm_q": 1 + randn(HEAD_DIM, std=0.1), "norm_k": 1 + randn(HEAD_DIM, std=0.1),
        })
    host = {
        "time_text_embed.timestep_embedder.linear_1.weight": randn(D, cfg.temb_dim).cpu().numpy(),
        "time_text_embed.timestep_embedder.linear_1.bias": randn(D).cpu().numpy(),
        "time_text_embed.timestep_embedder.linear_2.weight": randn(D, D).cpu().numpy(),
        "time_text_embed.timestep_embedder.linear_2.bias": randn(D).cpu().numpy(),
        "modulation.1.weight": randn(4 * D, D).cpu().numpy(),
        "norm_out.linear.weight": randn(D, D).cpu().numpy(),
    }
    img_in = randn(cfg.latent_ch, D)                      # B = W_img_in^T (64, D)
    proj_out = torch.zeros(D, 128, device=device)         # B = W_proj_out^T padded to 128 columns
    proj_out[:, :cfg.latent_ch] = randn(D, cfg.latent_ch)
    return {"blocks": blocks, "host": host, "img_in": img_in, "proj_out": proj_out}


def shard_weights(weights, cfg, rank, world):
    """Tensor-parallel shard `rank` of `world`: QKV columns and out-projection rows of this
    rank's heads (each head's q, k and v stay together), gate / proj units and down-projection rows of this rank's
    FFN units (interleaved 128-column tiles stay whole). Norm and host weights are replicated."""
    H, F, D = cfg.heads, cfg.ffn, cfg.hidden
    assert H % world == 0 and F % (64 * world) == 0, "heads and FFN units must split evenly (units by 64)"
    hl, fl = H // world, F // world
    c0, c1 = rank * hl * HEAD_DIM, (rank + 1) * hl * HEAD_DIM
    blocks = []
    for b in weights["blocks"]:
        qkv = b["qkv"]
        blocks.append({
            "qkv": torch.cat([qkv[:, c0:c1], qkv[:, D + c0:D + c1], qkv[:, 2 * D + c0:2 * D + c1]], 1).contiguous(),
            "o": b["o"][c0:c1].contiguous(),
            "gate": b["gate"][rank * fl:(rank + 1) * fl].contiguous(),
            "proj": b["proj"][rank * fl:(rank + 1) * fl].contiguous(),
            "down": b["down"][rank * fl:(rank + 1) * fl].contiguous(),
            "norm_q": b["norm_q"], "norm_k": b["norm_k"],
        })
    return {"blocks": blocks, "host": weights["host"], "img_in": weights["img_in"], "proj_out": weights["proj_out"]}


def interleave_up_torch(gate, proj):
    """[gate 64 | proj 64] per 128 columns of B = [Wgate^T, Wproj^T] (pack_weights.py:82-89)."""
    F, K = gate.shape
    B = torch.empty(K, F // 64, 2, 64, dtype=gate.dtype, device=gate.device)
    B[:, :, 0] = gate.t().reshape(K, F // 64, 64)
    B[:, :, 1] = proj.t().reshape(K, F // 64, 64)
    return B.reshape(K, 2 * F)


class DiT:
    """Resident packed weights + preallocated activations for one denoise step of config `cfg` on one GPU.

    tp = (rank, world, group): tensor-parallel over `world` GPUs with `weights` already sharded by shard_weights;
    the out-projection and down-projection write partial sums that are added up across the group (two reductions per
    block, the block being two sequential sublayers). reduce_dtype:
    "peer" (2 GPUs: the projection GEMM stores its bf16 partial into the other rank's memory as it computes it and
    the LayerNorm kernel adds the two: tp.PeerReduce; residual and LayerNorm replicated),
    "rs" (NCCL reduce-scatter of the bf16 partials, the residual + LayerNorm on this rank's M / world rows only -
    the residual stream stays sharded by rows - and an NCCL all-gather of the LayerNorm output, the next GEMM's A
    operand: the bytes of one all-reduce, and 1 / world of the LayerNorm work),
    "peer_rs" (the same three steps over peer memory on any number of GPUs: the projection GEMM stores each row
    block of its partial straight into the owning rank's memory as it computes it, the LayerNorm kernel of the owner
    adds the partials of its rows and stores its rows of the output into every rank's A operand: tp.PeerRS),
    "bf16" (one NCCL all-reduce of the bf16 partials, LayerNorm replicated), "fp32" (NCCL, fp32 partials) or "auto"
    (default: "peer_rs" when the rows split into multiples of 16 - per config-4 step 27.6 ms at 2 GPUs against 29.2
    for "peer" and 29.8 for "bf16", 17.8 ms at 4 GPUs against 22.2 for "bf16" and 22.7 for "rs" -, else "peer" at
    2 GPUs and "bf16" above).
    fuse_qkv: QK-RMSNorm + RoPE run in the QKV GEMM's epilogue (rl_qkv_linear) instead of rl_qkv_post after the
    GEMM."""

    def __init__(self, cfg, weights, device="cuda", tp=None, reduce_dtype="auto", fuse_qkv=True):
        if reduce_dtype not in ("auto", "peer", "peer_rs", "rs", "bf16", "fp32"):
            raise ValueError(f"reduce_dtype must be 'auto', 'peer', 'peer_rs', 'rs', 'bf16' or 'fp32', "
                             f"not {reduce_dtype!r}")
        if reduce_dtype == "auto":
            if tp and cfg.M % tp[1] == 0 and (cfg.M // tp[1]) % 16 == 0:
                reduce_dtype = "peer_rs"
            else:
                reduce_dtype = "peer" if tp and tp[1] == 2 else "bf16"
        if tp and reduce_dtype == "rs" and cfg.M % tp[1]:
            raise ValueError(f"reduce_dtype 'rs' needs M ({cfg.M}) divisible by the group size {tp[1]}")
        if tp and reduce_dtype == "peer_rs" and (cfg.M % tp[1] or (cfg.M // tp[1]) % 16):
            raise ValueError(f"reduce_dtype 'peer_rs' needs M / group size ({cfg.M} / {tp[1]}) to be a multiple "
                             f"of 16")
        self.reduce_dtype = reduce_dtype if tp else None
        self.reduce_f32 = reduce_dtype == "fp32"
        self.fuse_qkv = fuse_qkv   # False: the QKV GEMM and rl_qkv_post as two launches (the reference's two steps)
        self.cfg = cfg
        dev = torch.device(device)
        self.dev = dev
        self.tp = tp
        world = tp[1] if tp else 1
        D, M = cfg.hidden, cfg.M
        H, F = cfg.heads // world, cfg.ffn // world
        self.heads_local = H
        def pw(t, swiglu=False):     # float B (packed here) or an already resident PackedWeight (weights.load_packed)
            return t if isinstance(t, ops.PackedWeight) else ops.PackedWeight.from_float(t.to(dev), swiglu=swiglu)

        self.blocks = []
        for b in weights["blocks"]:
            up = b["up"] if "up" in b else interleave_up_torch(b["gate"], b["proj"])
            self.blocks.append({
                "qkv": pw(b["qkv"]), "o": pw(b["o"]), "up": pw(up, swiglu=True), "down": pw(b["down"]),
                "wq": (b["norm_q"] * C_LOG2).to(dev).float().contiguous(),
                "wk": b["norm_k"].to(dev).float().contiguous(),
            })
        self.img_in = pw(weights["img_in"])
        self.proj_out = pw(weights["proj_out"])
        self.host = weights["host"]
        # adaLN conditioning weights, resident in fp32 for the per-step glue on the GPU (set_t)
        te = "time_text_embed.timestep_embedder."

        def f32(name, required=True):
            a = self.host.get(name)
            if a is None:
                if required:
                    raise KeyError(f"host weight {name} missing")
                return None
            return torch.as_tensor(np.asarray(a, np.float32)).to(dev).contiguous()
        self.glue = {"l1w": f32(te + "linear_1.weight"), "l1b": f32(te + "linear_1.bias", False),
                     "l2w": f32(te + "linear_2.weight"), "l2b": f32(te + "linear_2.bias", False),
                     "mod": f32("modulation.1.weight"), "norm": f32("norm_out.linear.weight")}
        self.freqs = torch.from_numpy(HG.timestep_freqs()).to(dev)
        T = self.glue["l1w"].shape[0]
        if (self.glue["l1w"].shape[1] != 2 * self.freqs.numel() or self.glue["mod"].shape != (4 * D, T)
                or self.glue["norm"].shape[0] < D):
            raise ValueError("adaLN weights do not match the config")
        self.t_e = torch.empty(2, 2 * self.freqs.numel(), dtype=torch.float32, device=dev)
        self.t_h = torch.empty(2, T, dtype=torch.float32, device=dev)
        self.t_te = torch.empty(2, T, dtype=torch.float32, device=dev)
        self.t_mod = torch.empty(2, 4 * D, dtype=torch.float32, device=dev)
        self.t_out = torch.empty(2, self.glue["norm"].shape[0], dtype=torch.float32, device=dev)
        pad, shapes = HG.joint_layout(np.zeros(cfg.text, bool), n_target=cfg.image, grid=cfg.grid)
        self.rope_cs = torch.from_numpy(HG.rope(pad, shapes)).to(dev).contiguous()     # (M, 64, 2)
        bf = dict(dtype=torch.bfloat16, device=dev)
        # "rs" / "peer_rs": this rank's rows [r0, r0 + rows) of the residual stream and of the reduced branch /
        # LayerNorm output
        sharded = bool(tp) and reduce_dtype in ("rs", "peer_rs")
        self.rows, self.r0 = (M // world, tp[0] * (M // world)) if sharded else (M, 0)
        self.x = [torch.empty(self.rows, D, **bf) for _ in range(2)]
        self.c_sh = torch.empty(self.rows, D, **bf) if self.rows < M and reduce_dtype == "rs" else None
        self.a_sh = torch.empty(self.rows, D, **bf) if self.rows < M else None
        self.emb = torch.empty(M, D, **bf)
        self.a = torch.empty(M, D, **bf)
        self.qkv = torch.empty(M, 3 * H * HEAD_DIM, **bf)
        self.ldv = (M + 127) // 128 * 128
        self.q = torch.empty(H, M, 128, **bf)
        self.k = torch.empty(H, M, 128, **bf)
        self.vt = torch.empty(H, 128, self.ldv, **bf)
        self.o = torch.empty(M, H * HEAD_DIM, **bf)
        self.c = torch.empty(M, D, **bf)
        self.c32 = torch.empty(M, D, dtype=torch.float32, device=dev) if tp and self.reduce_f32 else None
        self.h = torch.empty(M, F, **bf)
        self.lat_dq = torch.empty(cfg.image, cfg.latent_ch, **bf)
        self.v = torch.empty(cfg.image, 128, dtype=torch.float32, device=dev)
        self.params = {k: torch.empty(2, 2, D, **bf) for k in ("first", "mlp", "attn", "out")}
        self.peer = self.peer_rs = None
        if tp and reduce_dtype == "peer":
            from . import tp as TP
            self.peer = TP.PeerReduce(tp[2], tp[0], tp[1], M, D, dev)
        if tp and reduce_dtype == "peer_rs":
            from . import tp as TP
            self.peer_rs = TP.PeerRS(tp[2], tp[0], tp[1], M, D, dev)
            self.a = self.peer_rs.a       # the gathered LayerNorm output lives where the other ranks can store it

    # --- per-step adaLN parameters (forward.py:231-238), computed on the GPU ---
    def set_t(self, sigma):
        """Timestep embedding -> modulation / norm_out -> the four bf16 LayerNorm parameter sets, as six small
        kernels on the current stream (the reference runs these products on the host: host_glue.py:31-48)."""
        D, g = self.cfg.hidden, self.glue
        s = torch.cuda.current_stream().cuda_stream
        T, half = self.t_h.shape[1], self.freqs.numel()
        t0 = float(np.float32(HG.model_t(sigma)) * np.float32(1000.0))
        ptr = lambda a: None if a is None else a.data_ptr()
        L.call("rl_sinusoidal_embed", t0, 0.0, self.freqs.data_ptr(), half, self.t_e.data_ptr(), s)
        L.call("rl_matvec_f32", g["l1w"].data_ptr(), T, 2 * half, self.t_e.data_ptr(), 2, ptr(g["l1b"]), 0,
               self.t_h.data_ptr(), s)
        L.call("rl_matvec_f32", g["l2w"].data_ptr(), T, T, self.t_h.data_ptr(), 2, ptr(g["l2b"]), 1,
               self.t_te.data_ptr(), s)
        L.call("rl_matvec_f32", g["mod"].data_ptr(), 4 * D, T, self.t_te.data_ptr(), 2, None, 1,
               self.t_mod.data_ptr(), s)
        L.call("rl_matvec_f32", g["norm"].data_ptr(), self.t_out.shape[1], T, self.t_te.data_ptr(), 2, None, 1,
               self.t_out.data_ptr(), s)
        L.call("rl_adaln_params", self.t_mod.data_ptr(), self.t_out.data_ptr(), self.t_out.shape[1], D,
               self.params["first"].data_ptr(),
               self.params["mlp"].data_ptr(), self.params["attn"].data_ptr(), self.params["out"].data_ptr(), s)

    def _linear(self, x, w, out, epi=L.RL_EPI_NONE, out_dtype=L.RL_BF16):
        M, K = x.shape
        dst = out if isinstance(out, int) else out.data_ptr()
        L.call("rl_linear_bfp16", x.data_ptr(), M, K, w.native.data_ptr(), w.N, None, epi, dst, out_dtype,
               torch.cuda.current_stream().cuda_stream)

    def _ln(self, x, br, params, xo, y, row0=0):
        """Residual + LayerNorm of rows [row0, row0 + len(x)) of the sequence (text rows use parameter row 1)."""
        M, D = x.shape
        bdt = L.RL_F32 if (br is not None and br.dtype == torch.float32) else L.RL_BF16
        split = min(max(self.cfg.text - row0, 0), M)
        L.call("rl_ln_mod", x.data_ptr(), None if br is None else br.data_ptr(), bdt, params.data_ptr(), M, D,
               split, None if xo is None else xo.data_ptr(), y.data_ptr(), None,
               torch.cuda.current_stream().cuda_stream)

    def embed(self, latents, text_states):
        """x = [text | img_in(latents)]; a = LN1 (forward.py:396-412 with g = 1 and a zero residual)."""
        cfg = self.cfg
        s = torch.cuda.current_stream().cuda_stream
        lat = latents.to(self.dev, torch.bfloat16).contiguous()
        L.call("rl_quantize_bfp16", lat.data_ptr(), L.RL_BF16, cfg.image, cfg.latent_ch, L.RL_ROWMAJOR, None,
               self.lat_dq.data_ptr(), s)
        self._linear(self.lat_dq, self.img_in, self.emb[cfg.text:])
        self.emb[:cfg.text].copy_(text_states.to(self.dev, torch.bfloat16))
        if self.a_sh is None:
            self._ln(self.emb, None, self.params["first"], self.x[0], self.a)
            return
        import torch.distributed as dist
        self._ln(self.emb[self.r0:self.r0 + self.rows], None, self.params["first"], self.x[0], self.a_sh, self.r0)
        dist.all_gather_into_tensor(self.a, self.a_sh, group=self.tp[2])

    def _branch_ln(self, x, w, xin, params, xo):
        """The out / down projection followed by the residual + LayerNorm; under tensor parallelism the partial
        projections are summed across the group first (in the LayerNorm kernel itself for reduce_dtype "peer")."""
        if self.peer_rs is not None:    # "peer_rs": the same three steps over peer memory, no collective kernel
            s = torch.cuda.current_stream().cuda_stream
            slot, epoch = self.peer_rs.next()
            self.peer_rs.gemm(x, w, slot, s)
            self.peer_rs.signal(slot, epoch, s)
            split = min(max(self.cfg.text - self.r0, 0), self.rows)
            self.peer_rs.ln_mod(xin, slot, epoch, params, split, xo, s)
            return
        if self.a_sh is not None:       # "rs": reduce-scatter, LayerNorm of this rank's rows, all-gather
            import torch.distributed as dist
            self._linear(x, w, self.c)
            dist.reduce_scatter_tensor(self.c_sh, self.c, group=self.tp[2])
            self._ln(xin, self.c_sh, params, xo, self.a_sh, self.r0)
            dist.all_gather_into_tensor(self.a, self.a_sh, group=self.tp[2])
            return
        if self.peer is None:
            self._ln(xin, self._branch(x, w), params, xo, self.a)
            return
        s = torch.cuda.current_stream().cuda_stream
        slot, epoch = self.peer.next()
        out, mirror = self.peer.part(slot)
        M, K = x.shape
        L.call("rl_linear_bfp16_partial", x.data_ptr(), M, K, w.native.data_ptr(), w.N, out, mirror, s)
        self.peer.signal(slot, epoch, s)
        self.peer.ln_mod(xin, slot, epoch, params, self.cfg.text, xo, self.a, s)

    def close(self):
        """Release the peer buffers of reduce_dtype "peer" / "peer_rs" (a collective: every rank of the group calls
        it)."""
        if self.peer is not None or self.peer_rs is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.dev)
            dist.barrier(group=self.tp[2])
            if self.peer_rs is not None:
                self.a = None
            for pr in (self.peer, self.peer_rs):
                if pr is not None:
                    pr.close()
            self.peer = self.peer_rs = None

    def _branch(self, x, w):
        """The out / down projection: bf16 on one GPU; partial sums all-reduced across the TP group."""
        if not self.tp:
            self._linear(x, w, self.c)
            return self.c
        import torch.distributed as dist
        if self.reduce_f32:
            self._linear(x, w, self.c32, out_dtype=L.RL_F32)
            dist.all_reduce(self.c32, group=self.tp[2])
            return self.c32
        self._linear(x, w, self.c)
        dist.all_reduce(self.c, group=self.tp[2])
        return self.c

    def block(self, i, last=False):
        cfg, b = self.cfg, self.blocks[i]
        s = torch.cuda.current_stream().cuda_stream
        M, H = cfg.M, self.heads_local
        if self.fuse_qkv:   # QK-RMSNorm + RoPE in the QKV GEMM's epilogue
            L.call("rl_qkv_linear", self.a.data_ptr(), M, self.a.shape[1], b["qkv"].native.data_ptr(), H, H,
                   self.rope_cs.data_ptr(), b["wq"].data_ptr(), b["wk"].data_ptr(), self.q.data_ptr(),
                   self.k.data_ptr(), self.vt.data_ptr(), self.ldv, s)
        else:
            self._linear(self.a, b["qkv"], self.qkv)
            L.call("rl_qkv_post", self.qkv.data_ptr(), self.rope_cs.data_ptr(), b["wq"].data_ptr(),
                   b["wk"].data_ptr(), M, H, self.q.data_ptr(), self.k.data_ptr(), self.vt.data_ptr(), self.ldv, s)
        L.call("rl_attention", self.q.data_ptr(), self.k.data_ptr(), self.vt.data_ptr(), self.ldv, H, M, M, M, None,
               1.0, self.o.data_ptr(), H * HEAD_DIM, s)
        self._branch_ln(self.o, b["o"], self.x[0], self.params["mlp"], self.x[1])
        self._linear(self.a, b["up"], self.h, epi=L.RL_EPI_SWIGLU)
        self._branch_ln(self.h, b["down"], self.x[1], self.params["out" if last else "attn"], self.x[0])

    def project(self):
        """proj_out on the image rows of a (= norm_out output) -> velocity (image, 64) float32 (forward.py:261-269)."""
        cfg = self.cfg
        self._linear(self.a[cfg.text:], self.proj_out, self.v, out_dtype=L.RL_F32)
        return self.v[:, :cfg.latent_ch]

    def forward(self, latents, text_states, sigma):
        """One denoise step's transformer: the velocity for `latents` (image, 64) at noise level `sigma`."""
        self.set_t(sigma)
        self.embed(latents, text_states)
        for i in range(self.cfg.blocks):
            self.block(i, last=(i == self.cfg.blocks - 1))
        return self.project()

    def denoise_step(self, latents, text_states, i, sigmas=HG.SIGMAS):
        """Euler step i of the distilled schedule (forward.py:58-61, 605, 616)."""
        v = self.forward(latents, text_states, sigmas[i])
        nxt = sigmas[i + 1] if i + 1 < len(sigmas) else 0.0
        return latents.to(self.dev, torch.float32) + (nxt - sigmas[i]) * v
