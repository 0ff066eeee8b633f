"""B200 attention hot path behind the reference's ComfyUI override API."""
