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
