"""Console entry: the DeepSeek-V3-shaped model (61 layers, MLA, 256 MXFP4 experts, grouped sigmoid top-8; random-init
weights). Two launches: the generation server on one B200 (the experts that do not fit in HBM on the CPU engine
through the mailbox), or the EP=8 layer benchmark with the experts split over the node's GPUs."""

MODEL = {
    'id': 'deepseek-v3', 'order': 20, 'name': 'DeepSeek-V3 shape (configs 3-5)', 'port': 18190, 'ready_timeout': 1800,
    'hardware': '1x B200 + host CPU engine, or 8x B200 over NVSwitch',
    'options': [
        {'key': 'mode', 'label': 'launch', 'default': 'serve',
         'choices': [['serve', 'generation server, 1 GPU, tiered experts'],
                     ['ep', 'EP layer benchmark over several GPUs']]},
        {'key': 'hot', 'label': 'GPU expert slots (serve)', 'default': '0.44',
         'choices': [['0.44', '44% of each layer (what one B200 holds)'], ['0.4', '40%'], ['0.25', '25%']]},
        {'key': 'gpus', 'label': 'GPUs (EP)', 'default': '8', 'choices': [['8', '8'], ['4', '4'], ['2', '2']]},
        {'key': 'tokens', 'label': 'tokens per rank (EP)', 'default': '4',
         'choices': [['4', '4 (32 requests over 8 GPUs)'], ['16', '16']]},
    ],
}


def build(options, port):
    """(argv, env) of the process for the chosen options."""
    if options.get('mode', 'serve') == 'serve':
        return (['python', '-m', 'xtier_b200.serve', '--model', 'deepseek-v3', '--hot', options['hot'],
                 '--port', str(port)], {})
    argv = ['python', '-m', 'torch.distributed.run', '--nnodes=1', f"--nproc-per-node={options['gpus']}",
            '--master-addr', '127.0.0.1', '--master-port', str(port), '-m', 'xtier_b200.tools.ep_bench',
            '--tokens', options['tokens']]
    return argv, {'NCCL_NVLS_ENABLE': '0'}
