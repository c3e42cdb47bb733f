"""Console entry: the DeepSeek-V3-shaped model (61 layers, 256 MXFP4 experts) with its experts split over 8 B200s (EP=8).
Listed for the EP benchmark tool; the generation server for this model is not wired yet (launches the EP layer
benchmark instead)."""

MODEL = {
    'id': 'deepseek-v3', 'order': 20, 'name': 'DeepSeek-V3 shape, EP=8 (config 3)', 'port': 18190, 'ready_timeout': 600,
    'hardware': '8x B200, NVSwitch',
    'options': [
        {'key': 'gpus', 'label': 'GPUs', 'default': '8', 'choices': [['8', '8'], ['4', '4'], ['2', '2']]},
        {'key': 'tokens', 'label': 'tokens per rank', 'default': '4',
         'choices': [['4', '4 (32 requests over 8 GPUs)'], ['16', '16']]},
    ],
}


def build(options, port):
    argv = ['python', '-m', 'torch.distributed.run', '--nnodes=1', f"--nproc-per-node={options['gpus']}",
            '--master-addr', '127.0.0.1', '--master-port', str(port), '-m', 'xtier_b200.tools.ep_bench',
            '--tokens', options['tokens']]
    return argv, {'NCCL_NVLS_ENABLE': '0'}
