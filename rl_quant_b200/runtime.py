"""InferenceRunner: rollout inference of a GLAD inference copy (qrt/runtime.py:63-275).

Modes (qrt/runtime.py:34-37, 83-84):
  "max-autotune" / "manual-graph": the fused forward is captured once per
      (batch, dtype, device) in a CUDA graph with static input/output buffers;
      each call copies the observations in and replays.
  "eager": the fused forward is launched directly each call.

The fused path needs the qrt full-mode layout (QuantCNN + QuantLinear on the
encoder and actor MLP). A model without it runs ``act_inference`` op by op.

Weight hand-over (qrt/runtime.py:195-271): ``refresh_quant`` requantises
every quantised layer in two launches (all QuantLinears in one table, the
QuantCNN in one); ``sync_weights_from`` adds one batched cast-copy of every
same-named parameter/buffer. Both are captured as one CUDA graph on first
use; buffers never move, so captured forwards stay valid.
"""
from __future__ import annotations

import warnings

import torch
import torch.nn as nn

from . import _native as N
from .fused import FusedActor, FusedActorCritic, FusedCritic, FusedUnsupported, ppo_epilogue
from .qconv import QuantCNN
from .qlinear import QuantLinear

_MODES = ("max-autotune", "manual-graph", "eager")


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return N.DTYPE_F16
    if t.dtype == torch.float32:
        return N.DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


class _Graph:
    """``fn`` captured over static input buffer(s): ``static_in`` is a tensor or a
    tuple of tensors; a call copies its arguments into them and replays."""

    def __init__(self, fn, static_in):
        self.static_in = static_in
        args = static_in if isinstance(static_in, tuple) else (static_in,)
        dev = args[0].device
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                fn(*args)
        torch.cuda.current_stream(dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = fn(*args)

    def __call__(self, *xs):
        args = self.static_in if isinstance(self.static_in, tuple) else (self.static_in,)
        for a, x in zip(args, xs):
            if x.data_ptr() != a.data_ptr():
                a.copy_(x)
        self.graph.replay()
        return self.out


class _HostPipe:
    """Captured forwards over ``lanes`` input/output buffer pairs for host
    observations. Step k uses lane k % lanes: its host-to-device copy runs on a
    copy stream once the lane's previous forward has read the input, the forward
    (graph replay) and the device-to-host copy of the means run on the current
    stream after the copy. With two lanes the copy of step k+1 overlaps the
    forward of step k; forwards stay in one stream, one after the other."""

    def __init__(self, make_graph, example_dev, lanes):
        dev = example_dev.device
        self.lanes = [make_graph(example_dev.clone()) for _ in range(lanes)]
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.in_ready = [torch.cuda.Event() for _ in range(lanes)]
        self.free = [torch.cuda.Event() for _ in range(lanes)]
        self.used = [False] * lanes
        self.i = 0

    def __call__(self, host_obs, out):
        j = self.i % len(self.lanes)
        self.i += 1
        g = self.lanes[j]
        cur = torch.cuda.current_stream(g.static_in.device)
        cs = self.copy_stream
        if self.used[j]:
            cs.wait_event(self.free[j])
        with torch.cuda.stream(cs):
            g.static_in.copy_(host_obs, non_blocking=True)
        self.in_ready[j].record(cs)
        cur.wait_event(self.in_ready[j])
        g.graph.replay()
        out.copy_(g.out, non_blocking=True)
        self.free[j].record(cur)
        self.used[j] = True
        return out


class InferenceRunner:
    def __init__(self, model, mode: str = "max-autotune", with_critic: bool = False,
                 clone_outputs: bool = False, host_lanes: int = 2, normalize: bool = True):
        """``normalize``: act/evaluate apply the model's own observation normalisers
        first, as qrt's InferenceRunner does (act_inference and f_val, qrt/runtime.py:
        98-106); False for observations that arrive normalised, as in qrt's integration
        (qrt/integration.py:128-136, which compiles the heads without them)."""
        if mode not in _MODES:
            raise ValueError(f"unknown mode: {mode}")
        if host_lanes < 1:
            raise ValueError("host_lanes must be >= 1")
        self.host_lanes = host_lanes
        self.normalize = normalize
        self._pipes: dict[tuple, _HostPipe] = {}
        if model.training:
            warnings.warn("[rl_quant_b200] model is in train mode; call model.eval() for rollouts")
        self.model = model
        self.mode = mode
        self.with_critic = with_critic
        self.clone_outputs = clone_outputs
        self._quant_layers = [m for m in model.modules() if m is not model and hasattr(m, "requantize_")]
        try:
            self._fused = FusedActor(model)
        except FusedUnsupported as e:
            self._fused = None
            warnings.warn(f"[rl_quant_b200] fused GLAD forward unavailable ({e}); running op by op")
        self._fused_critic = None
        if with_critic:
            try:
                self._fused_critic = FusedCritic(model)
            except FusedUnsupported as e:
                warnings.warn(f"[rl_quant_b200] fused GLAD critic unavailable ({e}); running op by op")
        self._graphs: dict[tuple, _Graph] = {}
        # Gumbel stream of train-mode rollouts: seed from torch's default generator
        self._gumbel_seed = int(torch.randint(0, 2 ** 62, (1,)).item())
        self._gumbel_offset = None
        # PPO.act sampling stream (Philox, its own seed) and the fused actor + critic
        self._ppo_seed = int(torch.randint(0, 2 ** 62, (1,)).item())
        self._ppo_rng = None
        self._fused_ac = None
        self._fused_ac_err = None
        self._g_refresh = None
        self._g_sync = None
        self._sync_items = None

    # -- forward functions ----------------------------------------------------------------
    @staticmethod
    def _apply_norm(norm, x):
        return x if norm is None or isinstance(norm, nn.Identity) else norm(x)

    def _act_fn(self, po):
        if self._fused is not None:
            if self.normalize:
                po = self._apply_norm(getattr(self.model, "actor_obs_normalizer", None), po)
            mean = torch.empty(po.shape[0], 29, dtype=torch.float32, device=po.device)
            if self.model.training:
                # train-mode rollouts keep the Gumbel top-k exploration (qrt/encoder_opt.py:87-91),
                # drawn inside the kernel; the device offset advances on every (replayed) call
                self._fused.run(po, mean, gumbel=self._gumbel_state(po.device))
            else:
                self._fused.run(po, mean)
            return mean
        if not self.normalize:
            enc, _, _, _ = self.model._encode_terrain(po)
            return self.model.actor(enc)
        return self.model.act_inference({"policy_obs": po})[0]

    def _val_fn(self, co):
        m = self.model
        c = self._apply_norm(getattr(m, "critic_obs_normalizer", None), co) if self.normalize else co
        if self._fused_critic is not None and co.shape[1] == self._fused_critic.P + 2079:
            value = torch.empty(co.shape[0], 1, dtype=torch.float32, device=co.device)
            # train-mode rollouts: the critic's Gumbel term is drawn in the kernel too
            self._fused_critic.run(c, value, gumbel=self._gumbel_state(co.device) if m.training else None)
            return value
        enc_fn = getattr(m, "_encode_terrain_orig", None) if co.shape[1] - 2079 != getattr(
            m, "actor_proprio_dim", -1) else None
        enc, _, _, _ = (enc_fn or m._encode_terrain)(c)
        return m.critic(enc)

    def _call(self, key, fn, *xs):
        if self.mode == "eager":
            return fn(*xs)
        k = (key,) + tuple((tuple(x.shape), x.dtype, x.device) for x in xs)
        g = self._graphs.get(k)
        if g is None:
            static = tuple(x.clone() for x in xs)
            g = self._new_graph(fn, static if len(static) > 1 else static[0])
            self._graphs[k] = g
        out = g(*xs)
        if not self.clone_outputs:
            return out
        return tuple(o.clone() for o in out) if isinstance(out, tuple) else out.clone()

    def _new_graph(self, fn, static):
        """Capture ``fn``; the warm-up runs of the capture leave the device noise
        counters (Gumbel offset, PPO sampling offset) as they found them."""
        saved = [(a, getattr(self, a).clone() if getattr(self, a) is not None else None)
                 for a in ("_gumbel_offset", "_ppo_rng")]
        g = _Graph(fn, static)
        for a, old in saved:
            t = getattr(self, a)
            if t is None:
                continue
            if old is not None and old.device == t.device:
                t.copy_(old)
            else:
                t.zero_()
        return g

    # -- PPO.act in one forward -------------------------------------------------------------
    def _gumbel_state(self, dev):
        if self._gumbel_offset is None or self._gumbel_offset.device != dev:
            self._gumbel_offset = torch.zeros(1, dtype=torch.int64, device=dev)
        return self._gumbel_seed, self._gumbel_offset

    def _ppo_fn(self, po, co, std_fn, norms):
        B, dev = po.shape[0], po.device
        mean = torch.empty(B, 29, dtype=torch.float32, device=dev)
        value = torch.empty(B, 1, dtype=torch.float32, device=dev)
        actions = torch.empty(B, 29, dtype=torch.float32, device=dev)
        log_prob = torch.empty(B, dtype=torch.float32, device=dev)
        sigma = torch.empty(B, 29, dtype=torch.float32, device=dev)
        train = self.model.training
        an, cn = norms
        if an is None and cn is None:
            # one read of the shared scan for both heads
            if train:
                self._fused_ac.run(po, co, mean, value, gumbel=self._gumbel_state(dev))
            else:
                self._fused_ac.run(po, co, mean, value)
        else:
            # normalised groups differ in their scans: each head loads (and normalises) its own
            self._fused.run(po, mean, gumbel=self._gumbel_state(dev) if train else None, obs_norm=an)
            self._fused_critic.run(co, value, obs_norm=cn, gumbel=self._gumbel_state(dev) if train else None)
        if self._ppo_rng is None or self._ppo_rng.device != dev:
            self._ppo_rng = torch.zeros(2, dtype=torch.int64, device=dev)
        ppo_epilogue(mean, std_fn(), self._ppo_seed, self._ppo_rng, actions, log_prob, sigma)
        return actions, value, log_prob, mean, sigma

    # -- public API (qrt/runtime.py:128-191) ------------------------------------------------
    @torch.inference_mode()
    def warmup(self, example_po, example_co=None, n_warmup: int = 3):
        for _ in range(n_warmup):
            self.act(example_po)
        if self.with_critic:
            if example_co is None:
                raise ValueError("warmup needs example_co when with_critic=True")
            for _ in range(n_warmup):
                self.evaluate(example_co)
        torch.cuda.synchronize()
        return self

    @torch.inference_mode()
    def act(self, policy_obs):
        """Actor forward -> action mean [B, num_actions] (fp32 holding the fp16 result)."""
        return self._call("act", self._act_fn, policy_obs)

    @torch.inference_mode()
    def act_host(self, host_obs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """``act`` for observations in host memory: the rows are copied straight into
        the captured graph's input buffer (pinned memory makes the copy asynchronous)
        and the means straight back into ``out`` (host [B, num_actions] fp32; pinned
        if allocated here). Returns ``out``; its copy completes on the current stream,
        so synchronise before reading it (and before rewriting ``host_obs``).
        Consecutive calls rotate over ``host_lanes`` captured forwards, so the input
        copy of one call overlaps the forward of the previous one."""
        if host_obs.is_cuda:
            raise ValueError("act_host takes host observations; use act for device tensors")
        dev = self._device()
        B = host_obs.shape[0]
        if out is None:
            out = torch.empty(B, 29, dtype=torch.float32, pin_memory=True)
        if self.mode == "eager":
            x = host_obs.to(dev, non_blocking=True)
            out.copy_(self._act_fn(x), non_blocking=True)
            return out
        k = ("act", tuple(host_obs.shape), host_obs.dtype, dev)
        pipe = self._pipes.get(k)
        if pipe is None:
            pipe = _HostPipe(lambda st: self._new_graph(self._act_fn, st), host_obs.to(dev), self.host_lanes)
            self._pipes[k] = pipe
        return pipe(host_obs, out)

    def check_status(self) -> None:
        """Raise ``DeviceStatusError`` if any fused forward launched since the previous
        check (directly or by a captured graph's replay) reported that a bounded
        device-side wait ran out; its outputs are then not valid. Reads and clears the
        status word of every workspace (one host synchronisation): call it once per PPO
        iteration, as ``accelerate_runner`` does before each update."""
        for f in (self._fused, self._fused_critic, self._fused_ac):
            if f is not None:
                f.check_status()

    def _device(self):
        for t in self.model.parameters():
            return t.device
        for t in self.model.buffers():
            return t.device
        return torch.device("cuda")

    @torch.inference_mode()
    def evaluate(self, critic_obs):
        if not self.with_critic:
            raise RuntimeError("evaluate needs InferenceRunner(with_critic=True)")
        return self._call("val", self._val_fn, critic_obs)

    @torch.inference_mode()
    def ppo_act(self, policy_obs, critic_obs, std: torch.Tensor | None = None,
                log_std: torch.Tensor | None = None, obs_norm: tuple | None = None):
        """One PPO.act transition (rsl_rl/algorithms/ppo.py:129-140) in one forward:
        the fused actor + critic over one read of the shared scan (train-mode Gumbel
        terms when the model is in train mode), then the Normal(mean, std) sample and
        its log-probability (glad_ppo_epilogue). Returns (actions [B,A], values [B,1],
        actions_log_prob [B], action_mean [B,A], action_sigma [B,A]), all fp32.
        ``std`` (or ``log_std``, exponentiated per call) defaults to the model's own
        parameter; captured modes read the given tensor in place on every call, so it
        must keep its storage (an nn.Parameter updated in place does).

        ``obs_norm=(actor_norm, critic_norm)``: rsl_rl EmpiricalNormalization modules of
        the two groups, applied in the kernels while the raw f32 rows load (their
        ``_mean``/``_var`` are read in place on every call). Without it the runner's
        ``normalize`` setting applies the model's own normalisers first."""
        if not self.with_critic:
            raise RuntimeError("ppo_act needs InferenceRunner(with_critic=True)")
        an, cn = obs_norm if obs_norm is not None else (None, None)
        an = None if isinstance(an, nn.Identity) else an
        cn = None if isinstance(cn, nn.Identity) else cn
        if obs_norm is None and self.normalize:
            m = self.model
            policy_obs = self._apply_norm(getattr(m, "actor_obs_normalizer", None), policy_obs)
            critic_obs = self._apply_norm(getattr(m, "critic_obs_normalizer", None), critic_obs)
        if an is not None or cn is not None:
            if self._fused is None or self._fused_critic is None:
                raise FusedUnsupported("ppo_act with observation normalisers needs the fused actor and critic")
            key = ("ppo", id(an), id(cn))
        else:
            key = ("ppo",)
            if self._fused_ac is None and self._fused_ac_err is None:
                try:
                    self._fused_ac = FusedActorCritic(self.model)
                except FusedUnsupported as e:
                    self._fused_ac_err = str(e)
            if self._fused_ac is None:
                raise FusedUnsupported(f"fused actor + critic unavailable: {self._fused_ac_err}")
        if std is None and log_std is None:
            if getattr(self.model, "noise_std_type", "scalar") == "log":
                log_std = self.model.log_std
            else:
                std = self.model.std
        if std is not None:
            src = std
            std_fn = lambda: src.float()  # noqa: E731
        else:
            src = log_std
            std_fn = lambda: torch.exp(src.float())  # noqa: E731
        key = key + (src.data_ptr(),)
        return self._call(key, lambda po, co: self._ppo_fn(po, co, std_fn, (an, cn)), policy_obs, critic_obs)

    @torch.inference_mode()
    def act_sample(self, policy_obs):
        mean = self.act(policy_obs)
        std = self.model.std if hasattr(self.model, "std") else torch.exp(self.model.log_std)
        return torch.normal(mean, std.to(mean.dtype).expand_as(mean))

    # -- weight hand-over --------------------------------------------------------------------
    def _requant_all(self):
        qls = [m for m in self._quant_layers if isinstance(m, QuantLinear) and m.act_mode != "dynamic_full"]
        if qls:
            for i in range(0, len(qls), 16):
                chunk = qls[i:i + 16]
                arr = (N.GladQLinearSrc * len(chunk))(*[q.requant_src() for q in chunk])
                N.check(N.load().glad_requant_qlinear(arr, len(chunk), N.stream_handle()), "requant")
        for m in self._quant_layers:
            if isinstance(m, QuantCNN):
                m.requantize_()
            elif not isinstance(m, QuantLinear):
                m.requantize_()

    def _graphed(self, attr, fn):
        g = getattr(self, attr)
        if g is None:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                fn()
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            setattr(self, attr, g)
        g.replay()

    @torch.inference_mode()
    def refresh_quant(self, use_graph: bool = True):
        """Requantise every quantised layer from its current weights."""
        if not self._quant_layers:
            return
        if not use_graph:
            self._requant_all()
            return
        self._graphed("_g_refresh", self._requant_all)

    @torch.inference_mode()
    def sync_weights_from(self, src_model, use_graph: bool = True):
        """Cast-copy every same-named parameter/buffer of ``src_model`` (the fp32
        master) into this copy, then requantise (qrt/runtime.py:224-271)."""
        if self._sync_items is None:
            for p in self.model.parameters():
                p.requires_grad_(False)
            dst = dict(self.model.named_parameters())
            dst.update(dict(self.model.named_buffers()))
            items, keep = [], []
            for name, s in list(src_model.named_parameters()) + list(src_model.named_buffers()):
                d = dst.get(name)
                if d is None or d.shape != s.shape or not d.is_floating_point() or not s.is_floating_point():
                    continue
                if not (d.is_contiguous() and s.is_contiguous()):
                    raise ValueError(f"{name}: sync needs contiguous tensors")
                items.append(N.GladCastCopy(s.data_ptr(), d.data_ptr(), d.numel(), _dt(s), _dt(d)))
                keep.append((s, d))
            self._sync_items = (N.GladCastCopy * len(items))(*items)
            self._sync_keep = keep

        def _do():
            if len(self._sync_items):
                N.check(N.load().glad_cast_copy(self._sync_items, len(self._sync_items), N.stream_handle()),
                        "sync cast-copy")
            self._requant_all()

        if not use_graph:
            _do()
            return
        self._graphed("_g_sync", _do)

    def __repr__(self):
        return (f"InferenceRunner(mode={self.mode}, with_critic={self.with_critic}, "
                f"fused={self._fused is not None}, quant_layers={len(self._quant_layers)})")
