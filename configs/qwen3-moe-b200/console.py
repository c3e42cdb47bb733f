"""Console entry: the Qwen3-style MoE (48 layers, 128 NVFP4 experts, 40 % hot) on one B200 with the CPU tier through the mailbox."""

MODEL = {
    'id': 'qwen3-moe', 'order': 10, 'name': 'Qwen3-style MoE 48L (config 2)', 'port': 18180, 'ready_timeout': 900,
    'hardware': '1x B200 + host CPU engine',
    'options': [
        {'key': 'hot', 'label': 'GPU hot slots', 'default': '0.4',
         'choices': [['0.4', '40% of each layer (config 2)'], ['0.6', '60%'], ['1.0', 'every expert on the GPU']]},
        {'key': 'threads', 'label': 'CPU engine workers', 'default': '0',
         'choices': [['0', 'all CPUs but two'], ['8', '8'], ['4', '4']]},
        {'key': 'adapt', 'label': 'adaptive hot slots', 'default': 'on', 'choices': [['on', 'on'], ['off', 'off']]},
        {'key': 'trace', 'label': 'route trace', 'default': 'off',
         'choices': [['off', 'off'], ['on', 'write /tmp/xtier-route-trace.bin (planner input)']]},
        {'key': 'decode', 'label': 'token choice', 'default': 'greedy',
         'choices': [['greedy', 'greedy (temperatures refused)'], ['sampling', 'temperature / top-p per request'],
                     ['recall', 'greedy + Recall copy drafts (speculative, in-memory record)']]},
        {'key': 'prefix', 'label': 'prefix reuse', 'default': 'on',
         'choices': [['on', 'a prompt extending the previous request reuses its KV'], ['off', 'every prompt cold']]},
    ],
}


def build(options, port):
    """(argv, env) of the server process for the chosen options."""
    argv = ['python', '-m', 'xtier_b200.serve', '--model', 'qwen3-moe', '--hot', options['hot'], '--port', str(port)]
    if options['decode'] == 'sampling':
        argv.append('--sampling')
    elif options['decode'] == 'recall':
        argv += ['--recall', 'memory']
    if options['prefix'] == 'off':
        argv.append('--no-prefix-cache')
    env = {'XTIER_THREADS': options['threads'], 'XTIER_CACHE_ADAPT': '1' if options['adapt'] == 'on' else '0'}
    if options['trace'] == 'on':
        env['XTIER_ROUTE_TRACE'] = '/tmp/xtier-route-trace.bin'
    return argv, env
