"""HRM-Text model family: layers, backbone, recurrent architectures and the LM head."""
