"""CUDA-graph execution of one GR00T control step (VLM prefill + Flow4 DiT).

The reference drives its patched model through `PreparedInferenceEngine.full`
(coexecution/libero/inference.py:43-73) and captures the action path in CUDA
graphs (coexecution/optimization/groot/action.py).  `ControlStep` does the
same for the whole step: inputs are copied into static device buffers, one
graph replays VLM prefill and the 4 Euler steps, and the actions come back.
Capture happens once, after a warm-up call that loads the library, builds
the activation tables and sets kernel attributes.
"""

import torch


class ControlStep:
    def __init__(self, policy, batch, *, device="cuda", graph=True, pin=True):
        self.policy = policy
        self.device = torch.device(device)
        vlm, dit = policy.backbone.config, policy.action_head.config
        self.static = [
            torch.zeros(batch, vlm.visual_tokens, vlm.hidden, device=self.device, dtype=torch.bfloat16),
            torch.zeros(batch, vlm.text_tokens, device=self.device, dtype=torch.long),
            torch.zeros(batch, 1, dit.state_dim, device=self.device, dtype=torch.bfloat16),
            torch.zeros(batch, dit.action_horizon, dit.action_dim, device=self.device, dtype=torch.bfloat16),
        ]
        self.host_out = torch.empty(
            batch, dit.action_horizon, dit.action_dim, dtype=torch.bfloat16, pin_memory=pin and torch.cuda.is_available()
        )
        self.output = None
        self.graph = None
        self.use_graph = graph
        self.stream = torch.cuda.Stream(self.device)

    def _run(self):
        return self.policy(*self.static)

    def load(self, inputs):
        for dst, src in zip(self.static, inputs):
            dst.copy_(src, non_blocking=True)

    @torch.inference_mode()
    def capture(self):
        """Warm up eagerly twice, then capture the step into one graph."""
        with torch.cuda.stream(self.stream):
            for _ in range(2):
                self.output = self._run()
        self.stream.synchronize()
        if self.use_graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self.output = self._run()
        return self

    @torch.inference_mode()
    def replay(self):
        """Device-resident step: inputs already in the static buffers."""
        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self.output = self._run()
        return self.output

    @torch.inference_mode()
    def step(self, inputs):
        """End-to-end step from host (pinned) tensors to host actions."""
        with torch.cuda.stream(self.stream):
            self.load(inputs)
            self.replay()
            self.host_out.copy_(self.output, non_blocking=True)
        self.stream.synchronize()
        return self.host_out

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.static)

    def d2h_bytes(self):
        return self.host_out.numel() * self.host_out.element_size()

    def release(self):
        self.graph = None
        self.output = None


class CoExecutionStep:
    """VLM prefill and the action head on two streams at once, as piR2's
    S1/S2 co-execution runs them (coexecution/run.py:33-105: the action
    head on its own stream reads the features the VLM last published, while
    the VLM computes the next features on another stream).

    Features live in two device slots.  Step k runs the action head for
    (state_k, noise_k) on the features of the previous observation (slot
    k % 2) and, concurrently, the VLM prefill of observation k into slot
    (k + 1) % 2; the two graphs (one per slot assignment) are captured once
    and replayed alternately, so no features are copied.  `prime(inputs)`
    fills the first slot with a plain VLM prefill.
    """

    def __init__(self, policy, batch, *, device="cuda", pin=True):
        self.policy = policy
        self.device = torch.device(device)
        vlm, dit = policy.backbone.config, policy.action_head.config
        tokens = vlm.visual_tokens + vlm.text_tokens
        self.static = [
            torch.zeros(batch, vlm.visual_tokens, vlm.hidden, device=self.device, dtype=torch.bfloat16),
            torch.zeros(batch, vlm.text_tokens, device=self.device, dtype=torch.long),
            torch.zeros(batch, 1, dit.state_dim, device=self.device, dtype=torch.bfloat16),
            torch.zeros(batch, dit.action_horizon, dit.action_dim, device=self.device, dtype=torch.bfloat16),
        ]
        self.slots = [
            torch.zeros(batch, tokens, vlm.hidden, device=self.device, dtype=torch.bfloat16) for _ in range(2)
        ]
        self.actions = torch.zeros(batch, dit.action_horizon, dit.action_dim, device=self.device, dtype=torch.bfloat16)
        self.host_out = torch.empty_like(self.actions, device="cpu", pin_memory=pin and torch.cuda.is_available())
        self.stream = torch.cuda.Stream(self.device)      # action head (S1) and the graph's origin
        self.vlm_stream = torch.cuda.Stream(self.device)  # VLM prefill (S2)
        self.graphs = [None, None]
        self.parity = 0

    def load(self, inputs):
        for dst, src in zip(self.static, inputs):
            dst.copy_(src, non_blocking=True)

    def _step(self, read, write):
        visual, ids, state, noise = self.static
        self.vlm_stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.vlm_stream):
            self.slots[write].copy_(self.policy.backbone(visual, ids))
        self.actions.copy_(self.policy.action_head.get_action(self.slots[read], state, noise))
        torch.cuda.current_stream(self.device).wait_stream(self.vlm_stream)

    @torch.inference_mode()
    def prime(self, inputs):
        """Publishes the features of `inputs` into the slot the next step reads."""
        with torch.cuda.stream(self.stream):
            self.load(inputs)
            self.slots[self.parity].copy_(self.policy.backbone(self.static[0], self.static[1]))
        self.stream.synchronize()

    @torch.inference_mode()
    def capture(self):
        with torch.cuda.stream(self.stream):
            for parity in (0, 1):
                self._step(parity, 1 - parity)
        self.stream.synchronize()
        for parity in (0, 1):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=self.stream):
                self._step(parity, 1 - parity)
            self.graphs[parity] = graph
        return self

    @torch.inference_mode()
    def replay(self):
        """One co-executed step on the static inputs; returns the actions."""
        with torch.cuda.stream(self.stream):
            self.graphs[self.parity].replay()
        self.parity ^= 1
        return self.actions

    @torch.inference_mode()
    def step(self, inputs):
        """Host inputs of observation k -> host actions for state k (on the
        features of observation k - 1); publishes observation k's features."""
        with torch.cuda.stream(self.stream):
            self.load(inputs)
            self.replay()
            self.host_out.copy_(self.actions, non_blocking=True)
        self.stream.synchronize()
        return self.host_out

    def h2d_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.static)

    def d2h_bytes(self):
        return self.host_out.numel() * self.host_out.element_size()

    def release(self):
        self.graphs = [None, None]
