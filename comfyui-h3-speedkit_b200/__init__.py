"""ComfyUI V3 entry point of the B200 build (the reference's __init__.py:4-15)."""


async def comfy_entrypoint():
    from comfy_api.latest import ComfyExtension
    from .h3_speedkit.nodes import make_nodes

    class H3SpeedKitExtension(ComfyExtension):
        async def get_node_list(self):
            return make_nodes()

    return H3SpeedKitExtension()
