"""ComfyUI V3 node for the B200 path; CUDA imports happen only on execution.

``H3SpeedKitOptimize`` keeps the reference's node id and schema
(h3_speedkit/nodes.py:26-40 of H3 SpeedKit): MODEL in, (MODEL, report) out,
with an ``enabled`` switch.  The other reference nodes (environment report,
video VAE, RGB8 decode, MP4 export, indexed gate) are outside this path.
"""


def _io():
    from comfy_api.latest import io
    return io


def make_nodes():
    io = _io()

    class H3SpeedKitOptimize(io.ComfyNode):
        @classmethod
        def define_schema(cls):
            return io.Schema(
                node_id="H3SpeedKitOptimize", display_name="H3 SpeedKit · Optimize DiT (B200)",
                category="H3 SpeedKit", inputs=[io.Model.Input("model"), io.Boolean.Input("enabled", default=True)],
                outputs=[io.Model.Output(), io.String.Output("report")])

        @classmethod
        def execute(cls, model, enabled=True, attention=None):
            if not enabled:
                return io.NodeOutput(model.clone(), "H3 SpeedKit disabled")
            from .runtime import patch_model
            patched = patch_model(model, attention=attention)
            return io.NodeOutput(patched, "B200 (sm_100a) backend installed. Execution logs report fallback reasons.")

    return [H3SpeedKitOptimize]
